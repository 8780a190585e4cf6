// matvec.cu -- decode-time dequant-dot matvecs y = W.x for .som Q8_0, GGML Q4_K
// and GGML Q6_K weights, on sm_100a.
//
// Replaces the reference's per-row SIMT kernels gm_matvec_q4k / gm_matvec_q80
// (lxdde/ports/nouveau/gemma_capa.cu:433-514) and the CPU kernels
// gemm::matvec_q4_k / matvec_q8_0 (crates/soso-llm-core/src/gemm.rs:295-461).
// Same block layouts, same per-sub-block algebra  d*sc*Sum(q*x) - dmin*m*Sum(x)
// (dequant.rs:172-191), f32 accumulation; the summation order differs (it is a
// parallel reduction), which the parity tests bound by tolerance.
//
// Structure (one kernel per format, same skeleton):
//  * grid = a multiple of the SM count; CTA i owns the contiguous row range
//    row_strip(rows, i, grid) -- whole rows, so no cross-CTA reduction.
//  * Prologue, before griddepcontrol.wait: one bulk L2 prefetch per 64 KiB of
//    the CTA's weight bytes.  With programmatic dependent launch this streams
//    the next matvec's weights while the previous kernel is still running.
//  * After the wait: x is staged once per CTA in shared memory, pre-scaled so
//    that a code isolated in place in a register (a subnormal bit pattern)
//    times the staged value is code*x*2^-60 exactly (see common.cuh).  Per
//    32-element chunk sums of x feed the -dmin*m / bias terms.
//  * 32 eight-lane workers per CTA; worker w owns the contiguous block range
//    row_strip(cta_blocks, w, 32) and processes one block per iteration
//    (each lane 1/8 of the block), accumulating per row.  Rows split between
//    workers are finished by a deterministic fixup in shared memory, so the
//    result does not depend on scheduling.
#pragma once
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "tc_mmv.cuh"
#include "sosob200.h"

namespace sb {

constexpr int MV_WARPS = 8;
constexpr int MV_THREADS = MV_WARPS * 32;
constexpr int MV_WORKERS = MV_THREADS / 8;

// -------------------------------------------------------------------- Q4_K
// Block: d f16 | dmin f16 | scales[12] | qs[128]  (layout.rs:63-64).
// Lane c (0..7) of a worker reads qs chunk c = bytes 16c..16c+15: pair p = c/2,
// low nibbles = sub-block 2p elements l0..l0+15 (l0 = 16*(c&1)), high nibbles =
// sub-block 2p+1 (dequant.rs:181-186: byte pair*32+l -> elems pair*64+l, +32).
// sums[i] = x[32i] + ... + x[32i+31], one warp per chunk, coalesced loads.
__device__ __forceinline__ void chunk_sums32(float *sums, const float *__restrict__ x, int nchunks)
{
    const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int i = threadIdx.x >> 5; i < nchunks; i += nw) {
        const float v = warp_sum(x[i * 32 + lane]);
        if (lane == 0) sums[i] = v;
    }
}

struct Q4K {
    static constexpr int BE = 256, BB = 144, U = 4;
    // smem: X2 float2[nb*128] (swizzled), sx float[nb*8]
    static __host__ __device__ size_t smem_bytes(int cols) { return (size_t)cols * 4 + (size_t)cols / 32 * 4; }

    static __device__ void stage(float *smem, const float *__restrict__ x, int cols)
    {
        const int nb = cols / 256;
        float2 *X2 = reinterpret_cast<float2 *>(smem);
        float *sx = smem + cols;
        for (int i = threadIdx.x; i < nb * 128; i += blockDim.x) {
            int b = i >> 7, p = (i >> 5) & 3, l = i & 31;
            int c = 2 * p + (l >> 4), j = (l & 15) >> 1;
            float lo = x[b * 256 + p * 64 + l], hi = x[b * 256 + p * 64 + 32 + l];
            // byte l of a 4-byte word sits at bits 8*(l&1) after the kernel's
            // optional >>16, low nibble there, high nibble 4 bits up.
            float slo = (l & 1) ? 0x1p81f : 0x1p89f, shi = (l & 1) ? 0x1p77f : 0x1p85f;
            X2[b * 128 + c * 16 + (((j ^ c) & 7) << 1) + (l & 1)] = make_float2(lo * slo, hi * shi);
        }
        chunk_sums32(sx, x, nb * 8);
    }

    struct Frag {
        uint4 hdr, qv;
    };
    static __device__ __forceinline__ void load(Frag &f, const uint8_t *__restrict__ blk, int c)
    {
        f.hdr = ldg_stream_v4(blk);
        f.qv = ldg_stream_v4(blk + 16 + c * 16);
    }

    static __device__ __forceinline__ float dot(const Frag &f, int c, int bc, const float *smem, int cols)
    {
        const uint4 hdr = f.hdr, qv = f.qv;
        const float4 *X4 = reinterpret_cast<const float4 *>(smem) + bc * 64 + c * 8;
        const float *sx = smem + cols;
        float2 acc = make_float2(0.0f, 0.0f);
        const uint32_t ws[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t w = ws[i], v = w >> 16;
            const float4 xa = X4[((2 * i) ^ c) & 7], xb = X4[((2 * i + 1) ^ c) & 7];
            acc = ffma2(make_float2(bits_f(w & 0xFu), bits_f(w & 0xF0u)), make_float2(xa.x, xa.y), acc);
            acc = ffma2(make_float2(bits_f(w & 0xF00u), bits_f(w & 0xF000u)), make_float2(xa.z, xa.w), acc);
            acc = ffma2(make_float2(bits_f(v & 0xFu), bits_f(v & 0xF0u)), make_float2(xb.x, xb.y), acc);
            acc = ffma2(make_float2(bits_f(v & 0xF00u), bits_f(v & 0xF000u)), make_float2(xb.z, xb.w), acc);
        }
        // 6-bit scales/mins of sub-blocks 2p, 2p+1: get_scale_min_k4
        // (dequant.rs:150-167) on four sub-blocks at once, one byte each.
        const int p = c >> 1;
        const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
        const uint32_t SC = p < 2 ? (s0 & 0x3F3F3F3Fu) : ((s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u));
        const uint32_t M = p < 2 ? (s1 & 0x3F3F3F3Fu) : (((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u));
        const int sh = (2 * p & 3) * 8;
        const float sc_lo = (float)((SC >> sh) & 0xFFu), sc_hi = (float)((SC >> (sh + 8)) & 0xFFu);
        const float m_own = (float)((M >> (sh + 8 * (c & 1))) & 0xFFu);
        const __half2 dd = *reinterpret_cast<const __half2 *>(&hdr.x);
        const float d = __low2float(dd) * TWO_P60, dmin = __high2float(dd);
        // the -dmin*m*Sum(x) term of sub-block 2p (even lane) or 2p+1 (odd lane)
        return d * sc_lo * acc.x + d * sc_hi * acc.y - dmin * m_own * sx[bc * 8 + 2 * p + (c & 1)];
    }
};

// -------------------------------------------------------------------- Q8_0
// .som block: f32 scale | 32 x i8 (layout.rs:57-59), 4-byte aligned.  Lane c
// reads code word c (codes 4c..4c+3).  Codes are offset to q+128 (xor 0x80)
// so they are non-negative bit patterns; 128*Sum(x) is removed per block.
struct Q80 {
    static constexpr int BE = 32, BB = 36, U = 8;
    // smem per 4-element group g (cols/4 groups, 8 floats each):
    //   X[4g..4g+3] pre-scaled, then the accumulator seed
    //   (-128*2^-60*(x0+x2), -128*2^-60*(x1+x3)) that removes the +128 offset
    //   inside the lane's own sum, before it can grow.
    static __host__ __device__ size_t smem_bytes(int cols) { return (size_t)cols / 4 * 32; }

    static __device__ void stage(float *smem, const float *__restrict__ x, int cols)
    {
        float4 *S = reinterpret_cast<float4 *>(smem);
        for (int g = threadIdx.x; g < cols / 4; g += blockDim.x) {
            const float x0 = x[4 * g], x1 = x[4 * g + 1], x2 = x[4 * g + 2], x3 = x[4 * g + 3];
            S[2 * g] = make_float4(x0 * 0x1p89f, x1 * 0x1p81f, x2 * 0x1p89f, x3 * 0x1p81f);
            S[2 * g + 1] = make_float4(-0x1p-53f * (x0 + x2), -0x1p-53f * (x1 + x3), 0.0f, 0.0f);
        }
    }

    struct Frag {
        uint32_t scale, w;
    };
    static __device__ __forceinline__ void load(Frag &f, const uint8_t *__restrict__ blk, int c)
    {
        f.scale = ldg_u32(blk);
        f.w = ldg_u32(blk + 4 + 4 * c);
    }

    static __device__ __forceinline__ float dot(const Frag &f, int c, int bc, const float *smem, int cols)
    {
        const uint32_t t = f.w ^ 0x80808080u, v = t >> 16;  // codes as q + 128
        const float4 *S = reinterpret_cast<const float4 *>(smem) + 2 * (bc * 8 + c);
        const float4 X = S[0], B = S[1];
        float2 acc = ffma2(make_float2(bits_f(t & 0xFFu), bits_f(t & 0xFF00u)), make_float2(X.x, X.y),
                           make_float2(B.x, B.y));
        acc = ffma2(make_float2(bits_f(v & 0xFFu), bits_f(v & 0xFF00u)), make_float2(X.z, X.w), acc);
        return __uint_as_float(f.scale) * TWO_P60 * (acc.x + acc.y);
    }
};

// -------------------------------------------------------------------- Q6_K
// GGML block: ql[128] | qh[64] | i8 sc[16] | f16 d  (gguf2som/src/lib.rs:1639-1661),
// 2-byte aligned.  Lane g (0..7) takes l = 4g..4g+3 of both 128-element halves
// n: words A = ql[64n+4g], B = ql[64n+32+4g], H = qh[32n+4g] give codes
//   Q1 (elems 128n+l)    = A lo | (H bits 0-1)<<4     scale sc[8n + g/4]
//   Q2 (elems 128n+32+l) = B lo | (H bits 2-3)<<4     scale sc[8n + g/4 + 2]
//   Q3 (elems 128n+64+l) = A hi | (H bits 4-5)<<4     scale sc[8n + g/4 + 4]
//   Q4 (elems 128n+96+l) = B hi | (H bits 6-7)<<4     scale sc[8n + g/4 + 6]
// codes are q+32 (unsigned); 32*Sum(x) over each 4-element group is removed.
struct Q6K {
    static constexpr int BE = 256, BB = 210, U = 2;
    // smem: X float4[nb][2][8][4] (Q1..Q4 values of element 4g+k), sx4 float4[nb][2][8]
    static __host__ __device__ size_t smem_bytes(int cols) { return (size_t)cols * 4 + (size_t)cols; }

    static __device__ void stage(float *smem, const float *__restrict__ x, int cols)
    {
        const int nb = cols / 256;
        float4 *X = reinterpret_cast<float4 *>(smem);
        float4 *S = reinterpret_cast<float4 *>(smem + cols);
        for (int i = threadIdx.x; i < nb * 64; i += blockDim.x) {
            int b = i >> 6, n = (i >> 5) & 1, g = (i >> 2) & 7, k = i & 3;
            const float *xb = x + b * 256 + n * 128 + 4 * g + k;
            float s = (k & 1) ? 0x1p81f : 0x1p89f;
            // bank-spread: element k of lane g lives in slot (k + g/2) & 3
            X[((b * 2 + n) * 8 + g) * 4 + ((k + (g >> 1)) & 3)] =
                make_float4(xb[0] * s, xb[32] * s, xb[64] * s, xb[96] * s);
        }
        for (int i = threadIdx.x; i < nb * 16; i += blockDim.x) {
            int b = i >> 4, n = (i >> 3) & 1, g = i & 7;
            const float *xb = x + b * 256 + n * 128 + 4 * g;
            float4 r;
            r.x = (xb[0] + xb[1]) + (xb[2] + xb[3]);
            r.y = (xb[32] + xb[33]) + (xb[34] + xb[35]);
            r.z = (xb[64] + xb[65]) + (xb[66] + xb[67]);
            r.w = (xb[96] + xb[97]) + (xb[98] + xb[99]);
            S[i] = r;
        }
    }

    struct Frag {
        uint32_t A[2], B[2], H[2], sa[2], sb[2];
        unsigned short d;
    };
    static __device__ __forceinline__ void load(Frag &f, const uint8_t *__restrict__ blk, int g)
    {
#pragma unroll
        for (int n = 0; n < 2; n++) {
            f.A[n] = ldg_u32_a2(blk + 64 * n + 4 * g);
            f.B[n] = ldg_u32_a2(blk + 64 * n + 32 + 4 * g);
            f.H[n] = ldg_u32_a2(blk + 128 + 32 * n + 4 * g);
            f.sa[n] = ldg_u32_a2(blk + 192 + 8 * n);
            f.sb[n] = ldg_u32_a2(blk + 196 + 8 * n);
        }
        f.d = ldg_u16(blk + 208);
    }

    static __device__ __forceinline__ float dot(const Frag &f, int g, int bc, const float *smem, int cols)
    {
        const float4 *X = reinterpret_cast<const float4 *>(smem) + bc * 64;
        const float4 *S = reinterpret_cast<const float4 *>(smem + cols) + bc * 16;
        const float d = __half2float(__ushort_as_half(f.d)) * TWO_P60;
        const int gi = (g >> 2) * 8;
        float total = 0.0f;
#pragma unroll
        for (int n = 0; n < 2; n++) {
            const uint32_t A = f.A[n], B = f.B[n], H = f.H[n], sa = f.sa[n], sb = f.sb[n];
            const uint32_t q[4] = {(A & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u),
                                   (B & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u),
                                   ((A >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u),
                                   ((B >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u)};
            float2 a12 = make_float2(0.0f, 0.0f), a34 = make_float2(0.0f, 0.0f);
            const float4 *Xn = X + (n * 8 + g) * 4;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float4 xv = Xn[(k + (g >> 1)) & 3];
                const int sh = (k & 2) ? 16 : 0;
                const uint32_t msk = (k & 1) ? 0x3F00u : 0x3Fu;
                a12 = ffma2(make_float2(bits_f((q[0] >> sh) & msk), bits_f((q[1] >> sh) & msk)),
                            make_float2(xv.x, xv.y), a12);
                a34 = ffma2(make_float2(bits_f((q[2] >> sh) & msk), bits_f((q[3] >> sh) & msk)),
                            make_float2(xv.z, xv.w), a34);
            }
            // i8 scales sc[8n + g/4 + {0,2,4,6}]
            const float sc1 = (float)(int8_t)(sa >> gi), sc2 = (float)(int8_t)(sa >> (gi + 16));
            const float sc3 = (float)(int8_t)(sb >> gi), sc4 = (float)(int8_t)(sb >> (gi + 16));
            const float4 s4 = S[n * 8 + g];
            // sum_i sc_i * (S_i - 32 * sx_i), with S_i carried at scale 2^-60
            total += sc1 * a12.x + sc2 * a12.y + sc3 * a34.x + sc4 * a34.y;
            total -= 0x1p-55f * (sc1 * s4.x + sc2 * s4.y + sc3 * s4.z + sc4 * s4.w);
        }
        return d * total;
    }
};

// ------------------------------------------------------------------ kernel
template <class F>
__global__ void __launch_bounds__(MV_THREADS) matvec_kernel(const uint8_t *__restrict__ W, int rows, int cols,
                                                            const float *__restrict__ x, float *__restrict__ y)
{
    extern __shared__ __align__(16) float smem[];
    __shared__ float seg_first[MV_WORKERS], seg_last[MV_WORKERS];

    __shared__ int wrange[MV_WORKERS + 1];
    const int nb = cols / F::BE;
    int r0, r1;
    row_strip(rows, blockIdx.x, gridDim.x, r0, r1);
    const int cb0 = r0 * nb, cb1 = r1 * nb;  // this CTA's blocks

#ifndef SB_NO_L2PF
    if (threadIdx.x < 32) prefetch_range_l2(W, (long long)cb0 * F::BB, (long long)cb1 * F::BB);
#endif
    if (threadIdx.x <= MV_WORKERS) {
        int s0, e0;
        row_strip(cb1 - cb0, threadIdx.x < MV_WORKERS ? threadIdx.x : MV_WORKERS - 1, MV_WORKERS, s0, e0);
        wrange[threadIdx.x] = cb0 + (threadIdx.x < MV_WORKERS ? s0 : e0);
    }
    griddep_wait();
    F::stage(smem, x, cols);
    __syncthreads();
    griddep_launch();

    const int worker = threadIdx.x >> 3, c = threadIdx.x & 7;
    const int wb0 = wrange[worker], wb1 = wrange[worker + 1];

    if (wb0 < wb1) {
        int row = wb0 / nb;
        int bc = wb0 - row * nb;
        int seg_start = wb0;
        float acc = 0.0f;
        const uint8_t *rowp = W + (size_t)row * nb * F::BB;
        for (int b = wb0; b < wb1; b += F::U) {
            // issue the loads of up to U blocks before any of them is used
            typename F::Frag fr[F::U];
#pragma unroll
            for (int u = 0; u < F::U; u++)
                if (b + u < wb1) F::load(fr[u], W + (size_t)(b + u) * F::BB, c);
#pragma unroll
            for (int u = 0; u < F::U; u++) {
                if (b + u < wb1) {
                    acc += F::dot(fr[u], c, bc, smem, cols);
                    if (++bc == nb || b + u + 1 == wb1) {
                        const float v = warp8_sum(acc);
                        const bool starts = seg_start == row * nb, ends = bc == nb;
                        if (c == 0) {
                            if (starts && ends) y[row] = v;
                            else if (starts) seg_last[worker] = v;  // owner of a row that continues
                            else seg_first[worker] = v;             // continuation (middle or last piece)
                        }
                        acc = 0.0f;
                        bc = 0;
                        row++;
                        seg_start = b + u + 1;
                    }
                }
            }
        }
        (void)rowp;
    }
    __syncthreads();
    // Deterministic fixup of rows split between workers: the worker holding a
    // row's first block adds the following workers' pieces in order.
    if (threadIdx.x < MV_WORKERS) {
        const int w = threadIdx.x;
        const int a0 = wrange[w], a1 = wrange[w + 1];
        if (a0 < a1) {
            const int last_row = (a1 - 1) / nb;
            const int row_end = (last_row + 1) * nb;
            if (a1 < row_end && last_row * nb >= a0) {
                float total = seg_last[w];
                for (int w2 = w + 1; w2 < MV_WORKERS; w2++) {
                    const int b0 = wrange[w2], b1 = wrange[w2 + 1];
                    if (b0 >= b1) break;
                    total += seg_first[w2];
                    if (b1 >= row_end) break;
                }
                y[last_row] = total;
            }
        }
    }
}

template <class F>
static int launch_matvec(const void *w, size_t rows, size_t cols, const float *x, float *y, int pdl,
                         cudaStream_t stream)
{
    static int num_sms[64];
    static size_t smem_set[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -3;
    if (!num_sms[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        num_sms[dev] = n > 0 ? n : 148;
    }
    const size_t smem = F::smem_bytes((int)cols);
    if (smem > 48 * 1024 && smem > smem_set[dev]) {
        if (cudaFuncSetAttribute(matvec_kernel<F>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return -3;
        smem_set[dev] = smem;
    }
    // as many CTAs per SM as shared memory allows (registers cap it at 3), never more CTAs than rows
    int per_sm = smem <= 64 * 1024 ? 3 : smem <= 100 * 1024 ? 2 : 1;
    long long grid = (long long)num_sms[dev] * per_sm;
    if ((long long)rows < grid) grid = (long long)rows;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(MV_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, matvec_kernel<F>, (const uint8_t *)w, (int)rows, (int)cols, x, y);
    return e == cudaSuccess ? 0 : -4;
}

}  // namespace sb

extern "C" size_t sbk_row_bytes(uint8_t dtype, size_t cols)
{
    size_t e, b;
    switch (dtype) {
    case SB_DTYPE_Q8_0: e = 32; b = 36; break;
    case SB_DTYPE_Q4_K: e = 256; b = 144; break;
    case SB_DTYPE_Q6_K: e = 256; b = 210; break;
    case SB_DTYPE_Q6_K_P: return (cols == 0 || cols % 256) ? 0 : sb::tcmv::q6k_packed_row_bytes(cols);
    case SB_DTYPE_Q8_0_R: return (cols == 0 || cols % 32) ? 0 : sb::tcmv::q80_row_bytes_padded(cols);
    case SB_DTYPE_F32: return cols * 4;
    default: return 0;
    }
    if (cols == 0 || cols % e) return 0;
    return cols / e * b;
}

namespace sb {
// Per (device, stream) workspace for the split-row kernels, grown on demand and
// zero-initialised.  Growing allocates: make the first call of a shape outside
// stream capture.
struct WsCache {
    std::mutex mu;
    std::unordered_map<unsigned long long, std::pair<void *, size_t>> m;
};
static WsCache g_ws;

static void *stream_ws(cudaStream_t s, size_t bytes)
{
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long key = ((unsigned long long)dev << 56) ^ (unsigned long long)(uintptr_t)s;
    std::lock_guard<std::mutex> lk(g_ws.mu);
    auto &e = g_ws.m[key];
    if (e.second >= bytes) return e.first;
    if (e.first) {
        cudaStreamSynchronize(s);
        cudaFree(e.first);
    }
    e.first = nullptr;
    e.second = 0;
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    if (cudaMalloc(&e.first, want) != cudaSuccess) return nullptr;
    // zeroed on the launching stream itself, so that the first kernel on it is ordered after
    // the clear (a plain cudaMemset runs on the legacy stream, which a non-blocking stream
    // does not wait for)
    if (cudaMemsetAsync(e.first, 0, want, s) != cudaSuccess) {
        cudaFree(e.first);
        e.first = nullptr;
        return nullptr;
    }
    e.second = want;
    return e.first;
}

static int num_sms_cached()
{
    static int n[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!n[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        n[dev] = v > 0 ? v : 148;
    }
    return n[dev];
}
}  // namespace sb

namespace sb {
// Up to MAXB matrices of format F per launch of the tensor-core kernel; with
// `fallback`, a chunk the kernel does not take runs matrix by matrix through
// sbk_matvec, else it is rejected (-5).
template <class F, class FB = Q4K>
static int tc_matvec_batch(const sbk_mv_op *ops, size_t n, int pdl, cudaStream_t s, bool fallback,
                           const tcmv::XSrc *xs = nullptr, const grp::Pub *pub = nullptr,
                           const grp::Wait *wait = nullptr, bool pairs = false)
{
    if (pairs) fallback = false;
    if ((pub && pub->n) || (wait && wait->n)) fallback = false;
    if (xs && xs->mode != tcmv::XS_PLAIN) fallback = false;  // the CUDA-core kernel has no fused input forms
    const int grid = num_sms_cached();
    for (size_t i0 = 0; i0 < n; i0 += tcmv::MAXB) {
        const size_t nb = n - i0 < (size_t)tcmv::MAXB ? n - i0 : (size_t)tcmv::MAXB;
        tcmv::MatOp mo[tcmv::MAXB];
        bool ok = true;
        for (size_t i = 0; i < nb; i++) {
            const sbk_mv_op &o = ops[i0 + i];
            if (!o.w || !o.x || !o.y || !o.rows || ((uintptr_t)o.w & 15) || ((uintptr_t)o.x & 15) ||
                sbk_row_bytes(F::DTYPE, o.cols) == 0)
                return -1;
            mo[i] = tcmv::MatOp{o.w, (int)o.rows, (int)o.cols, o.x, o.y};
            ok = ok && o.rows < (1u << 24);
        }
        if (ok && tcmv::fits<F>(mo, (int)nb, grid)) {
            void *ws = stream_ws(s, tcmv::ws_bytes(grid));
            if (!ws) return -3;
            const int rc = tcmv::launch_batch<F>(mo, (int)nb, ws, grid, pdl, s, xs, pub, wait, pairs);
            if (rc) return rc;
        } else if (fallback) {
            for (size_t i = 0; i < nb; i++) {
                const sbk_mv_op &o = ops[i0 + i];
                const int rc = launch_matvec<FB>(o.w, o.rows, o.cols, o.x, o.y, pdl, s);
                if (rc) return rc;
            }
        } else {
            return -5;
        }
    }
    return 0;
}
}  // namespace sb

extern "C" int sbk_matvec(uint8_t dtype, const void *w, size_t rows, size_t cols, const float *x, float *y,
                          int pdl, void *stream)
{
    if (!w || !x || !y || rows == 0 || rows > (1u << 30)) return -1;
    if (!sbk_row_bytes(dtype, cols) || cols > 65536) return -1;
    if ((unsigned long long)rows * (cols / 32) >= (1ull << 31)) return -1;  // block indices are 32-bit
    if (((uintptr_t)w & 15) || ((uintptr_t)x & 15)) return -2;
    cudaStream_t s = (cudaStream_t)stream;
    const sbk_mv_op op{w, rows, cols, x, y};
    switch (dtype) {
    case SB_DTYPE_Q4_K: return sb::tc_matvec_batch<sb::tcmv::Q4K>(&op, 1, pdl, s, true);
    case SB_DTYPE_Q6_K_P: return sb::tc_matvec_batch<sb::tcmv::Q6KP>(&op, 1, pdl, s, false);
    case SB_DTYPE_Q8_0:
        // rows of a multiple of 128 weights are 16-byte aligned: the tensor-core kernel reads them
        if (cols % 128 == 0) return sb::tc_matvec_batch<sb::tcmv::Q80, sb::Q80>(&op, 1, pdl, s, true);
        return sb::launch_matvec<sb::Q80>(w, rows, cols, x, y, pdl, s);
    case SB_DTYPE_Q8_0_R: return sb::tc_matvec_batch<sb::tcmv::Q80, sb::Q80>(&op, 1, pdl, s, false);
    case SB_DTYPE_Q6_K: return sb::launch_matvec<sb::Q6K>(w, rows, cols, x, y, pdl, s);
    }
    return -1;
}

extern "C" int sbk_matvec_batch(uint8_t dtype, const sbk_mv_op *ops, size_t n, int pdl, void *stream)
{
    if (!ops || n == 0) return -1;
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == SB_DTYPE_Q4_K) return sb::tc_matvec_batch<sb::tcmv::Q4K>(ops, n, pdl, s, true);
    if (dtype == SB_DTYPE_Q6_K_P) return sb::tc_matvec_batch<sb::tcmv::Q6KP>(ops, n, pdl, s, false);
    if (dtype == SB_DTYPE_Q8_0_R) return sb::tc_matvec_batch<sb::tcmv::Q80, sb::Q80>(ops, n, pdl, s, false);
    if (dtype == SB_DTYPE_Q8_0) {
        bool aligned = true;
        for (size_t i = 0; i < n; i++) aligned = aligned && ops[i].cols % 128 == 0;
        if (aligned) return sb::tc_matvec_batch<sb::tcmv::Q80, sb::Q80>(ops, n, pdl, s, true);
    }
    for (size_t i = 0; i < n; i++) {
        const int rc = sbk_matvec(dtype, ops[i].w, ops[i].rows, ops[i].cols, ops[i].x, ops[i].y, pdl, stream);
        if (rc) return rc;
    }
    return 0;
}

namespace sb {
// sbk_matvec_batch_x with the group forms: wait for an exchange point before reading the
// input, and/or publish the (single) matrix's rows to the group (engine.cuh).
// pairs: one matrix whose rows are 16-row groups of a gate and an up projection in turn;
// its output is silu(gate) * up (rows / 2 entries).
inline int matvec_batch_group(uint8_t dtype, const sbk_mv_op *ops, size_t n, const tcmv::XSrc &x,
                              const grp::Pub *pub, const grp::Wait *wait, cudaStream_t s, bool pairs = false)
{
    if (dtype == SB_DTYPE_Q4_K) return tc_matvec_batch<tcmv::Q4K>(ops, n, 1, s, false, &x, pub, wait, pairs);
    if (dtype == SB_DTYPE_Q6_K_P) return tc_matvec_batch<tcmv::Q6KP>(ops, n, 1, s, false, &x, pub, wait, pairs);
    if (dtype == SB_DTYPE_Q8_0_R)
        return tc_matvec_batch<tcmv::Q80, Q80>(ops, n, 1, s, false, &x, pub, wait, pairs);
    return -5;
}
}  // namespace sb

extern "C" int sbk_matvec_batch_x(uint8_t dtype, const sbk_mv_op *ops, size_t n, const sbk_xsrc *xs, int pdl,
                                  void *stream)
{
    if (!ops || n == 0 || !xs) return -1;
    const sb::tcmv::XSrc x{xs->res, xs->norm_w, xs->h_out, xs->eps, xs->mode, xs->ys, xs->yw, xs->ny, xs->ystride};
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == SB_DTYPE_Q4_K) return sb::tc_matvec_batch<sb::tcmv::Q4K>(ops, n, pdl, s, true, &x);
    if (dtype == SB_DTYPE_Q6_K_P) return sb::tc_matvec_batch<sb::tcmv::Q6KP>(ops, n, pdl, s, false, &x);
    if (dtype == SB_DTYPE_Q8_0_R) return sb::tc_matvec_batch<sb::tcmv::Q80, sb::Q80>(ops, n, pdl, s, false, &x);
    if (dtype == SB_DTYPE_Q8_0) {
        for (size_t i = 0; i < n; i++)
            if (ops[i].cols % 128) return -5;  // unaligned rows: pad them first (sbk_q80_pad)
        return sb::tc_matvec_batch<sb::tcmv::Q80, sb::Q80>(ops, n, pdl, s, false, &x);
    }
    return -5;
}

extern "C" int sbk_q80_pad(const void *src, size_t rows, size_t cols, void *dst, void *stream)
{
    if (!src || !dst || !rows || cols % 32 || cols > (1u << 24) || rows > (1u << 30)) return -1;
    if ((uintptr_t)dst & 15) return -2;
    const int rb = (int)(cols / 32 * 36), rbp = (int)sb::tcmv::q80_row_bytes_padded(cols);
    const long long n = (long long)rows * rbp;
    sb::tcmv::q80_pad_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint8_t *>(src), (long long)rows, rb, reinterpret_cast<uint8_t *>(dst), rbp);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int sbk_q6k_pack(const void *src, size_t rows, size_t cols, void *dst, void *stream)
{
    if (((uintptr_t)dst & 15)) return -2;
    return sb::tcmv::q6k_pack(src, rows, cols, dst, (cudaStream_t)stream);
}

extern "C" int sbk_num_sms(int device)
{
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
    return n;
}

extern "C" int sbk_take_device_error(int device, uint32_t *code)
{
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return -1;
    unsigned int v = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, sb::g_dev_error, sizeof(v));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(sb::g_dev_error, &zero, sizeof(zero));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return -2;
    if (code) *code = v;
    return 0;
}
