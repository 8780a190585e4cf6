// prefill.cuh -- batched prefill GEMM on the sm_100a tensor cores (tcgen05):
//   Y[n x rows] = X[n x cols] . W^T,  W quantized (reference block layouts), X f32.
//
// Replaces the reference's block-prefill GEMM `iq_matmul_mma` (lxdde/ports/nouveau/
// matvec_iq.cu:731-816, :966: weights decoded to f16 in shared memory, mma.sync
// m16n8k16) and the CPU batch kernel `matvec_q4_k_batch` (crates/soso-llm-core/src/
// gemm.rs:495-546) behind GpuDispatch::matmul (crates/soso-llm-core/src/gpu.rs:443-455).
//
// Shape of the work: the MMA is D[128 x 256] += A[128 x 16] . B[256 x 16]^T with
// A = a 128-row tile of W dequantised to bf16 in shared memory and B = a 256-token
// tile of X (bf16, brought in by TMA with the 128-byte swizzle), both K-major, D
// (f32) in tensor memory: 256 of its 512 columns.  One CTA owns one (128 rows x 256
// tokens) output tile over the whole K, so every weight byte is read and
// dequantised once per 256 tokens.
//
// Warp roles (10 warps):
//   warp 0     TMA producer: raw weight blocks (one 256-column block column per
//              4 stages) and the X tile of every 64-column stage
//   warp 1     owns the tensor-memory allocation; one elected lane issues the
//              tcgen05.mma of a stage (4 x K16) and commits it to the stage's
//              `empty` barrier, and after the last stage to `acc_full`
//   warps 2-9  dequantise: two threads per weight row of the tile, one 64-column
//              stage at a time (Q4_K: one byte pair, sub-block 2p or 2p+1 each),
//              writing 16-bit rows in the 128-byte-swizzled K-major layout the MMA
//              descriptor describes; then the epilogue: tcgen05.ld of their
//              32 lanes (warp w reads lanes 32*(w%4)..; the two warps of a lane
//              quadrant split the columns), stores of Y (a warp writes 32
//              consecutive rows of one token: coalesced).
// Every mbarrier wait is bounded and reports through the device error word; the
// tensor memory is always freed after the last commit has landed.
#pragma once
#include <cuda_bf16.h>

#include "tc_common.cuh"

namespace sb {
namespace pf {

constexpr int BM = 128;       // weight rows per tile (MMA M)
constexpr int BN = 256;       // tokens per tile (MMA N)
constexpr int BK = 64;        // columns per stage: one 128-byte swizzle atom of bf16
constexpr int NST = 3;        // stages in flight
constexpr int RAWK = 256;     // columns per raw weight block column (one Q4_K block)
constexpr int NRAW = 2;       // raw weight block columns in flight
constexpr int NDQ = 8;        // dequantising / epilogue warps: two threads per weight row
constexpr int THREADS = (2 + NDQ) * 32;
constexpr int X_BYTES = BN * BK * 2;   // 32 KiB
constexpr int W_BYTES = BM * BK * 2;   // 16 KiB
constexpr int TMEM_COLS = 256;
constexpr unsigned WAIT = 1u << 22;  // bounded waits: a few seconds at most

// Q4_K raw tile: 128 rows x one 144-byte block
constexpr int RAW_ROWB = 144;
constexpr int RAW_BYTES = BM * RAW_ROWB;  // 18 KiB

struct Smem {
    uint8_t *x0, *w0, *raw0;  // stage i at x0 + i X_BYTES, w0 + i W_BYTES (1024-aligned), raw0 + i RAW_BYTES
    __device__ uint8_t *x(int i) const { return x0 + i * X_BYTES; }
    __device__ uint8_t *w(int i) const { return w0 + i * W_BYTES; }
    __device__ uint8_t *raw(int i) const { return raw0 + i * RAW_BYTES; }
    uint64_t *x_full, *w_full, *st_empty, *raw_full, *raw_empty, *acc_full;
    uint32_t *tmem_addr;
};

inline size_t smem_bytes() { return 1024 + NST * (X_BYTES + W_BYTES) + NRAW * RAW_BYTES + 256; }

__device__ __forceinline__ Smem carve(uint8_t *raw_base)
{
    Smem s;
    // aligned by an offset from the shared array, which keeps the accesses in the shared window
    uint8_t *b = raw_base + ((1024u - (tcmv::smem_u32(raw_base) & 1023u)) & 1023u);
    s.x0 = b;
    b += NST * X_BYTES;
    s.w0 = b;
    b += NST * W_BYTES;
    s.raw0 = b;
    b += NRAW * RAW_BYTES;
    uint64_t *bar = reinterpret_cast<uint64_t *>(b);
    s.x_full = bar;
    s.w_full = bar + NST;
    s.st_empty = bar + 2 * NST;
    s.raw_full = bar + 3 * NST;
    s.raw_empty = bar + 3 * NST + NRAW;
    s.acc_full = bar + 3 * NST + 2 * NRAW;
    s.tmem_addr = reinterpret_cast<uint32_t *>(bar + 3 * NST + 2 * NRAW + 1);
    return s;
}

// K-major, 128-byte swizzled operand tile: rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(const void *tile)
{
    const uint64_t addr = (uint64_t)tcmv::smem_u32(tile);
    return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: D f32, A and B both bf16 (F16 = false) or both f16,
// both K-major, M = 128, N = 256.
template <bool F16>
__host__ __device__ constexpr uint32_t idesc()
{
    return (1u << 4) | ((F16 ? 0u : 1u) << 7) | ((F16 ? 0u : 1u) << 10) | ((uint32_t)(BN >> 3) << 17) |
           ((uint32_t)(BM >> 4) << 24);
}

template <bool F16>
__device__ __forceinline__ void mma_16bit(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t acc)
{
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc<F16>()), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     tcmv::smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32])
{
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Two values as 16-bit operands (round to nearest even), a in the low half (lower column).
template <bool F16>
__device__ __forceinline__ uint32_t pack16(float a, float b)
{
    if (F16) {
        const __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&h);
    }
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Codes as exact floats, two at a time: prmt puts byte j of v into the low mantissa byte of
// 2^23 (0x4B000000), i.e. the float 2^23 + byte; one packed f32x2 add of -(2^23 + bias)
// leaves byte - bias exactly (bias 128 for a signed byte whose sign bit was flipped).
__device__ __forceinline__ uint32_t prmt_f(uint32_t v, uint32_t sel)
{
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(v), "r"(0x4B000000u), "r"(sel));
    return d;
}
__device__ __forceinline__ uint64_t f2(uint32_t lo, uint32_t hi)
{
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
    return d;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// bytes (j0, j1) of v as floats minus the bias held (negated, twice) in nbias2
__device__ __forceinline__ uint64_t codes2(uint32_t v, uint32_t sel0, uint32_t sel1, uint64_t nbias2)
{
    return add_f32x2(f2(prmt_f(v, sel0), prmt_f(v, sel1)), nbias2);
}
__device__ __forceinline__ uint64_t dup2(float x)
{
    return f2(__float_as_uint(x), __float_as_uint(x));
}
template <bool F16>
__device__ __forceinline__ uint32_t pack16x2(uint64_t w)
{
    return pack16<F16>(__uint_as_float((uint32_t)w), __uint_as_float((uint32_t)(w >> 32)));
}
// prmt selectors: byte j of v, then bytes 4, 4, 7 of 0x4B000000 (0, 0, 0x4B)
constexpr uint32_t SEL_B0 = 0x7440u, SEL_B1 = 0x7441u, SEL_B2 = 0x7442u, SEL_B3 = 0x7443u;

// Q4_K, one byte pair p of the block in `blk` (144 bytes), nibble half h: the 32 weights of
// sub-block 2p + h (h = 0: low nibbles, columns 0..31 of the stage; 1: high nibbles,
// columns 32..63) as d*sc*q - dmin*m (crates/sosomodel/src/dequant.rs:150-248), rounded to
// the operand type and written into this row of the swizzled stage tile.
template <bool F16>
__device__ __forceinline__ void q4k_half_to_16(const uint8_t *blk, int p, int h, uint8_t *row, int r)
{
    // the block's 16-byte head in one load: d, dmin (f16), then the 12 packed scale bytes
    const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
    const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
    auto sc = [&](int k) {  // scale byte k (selects, not an indexed array: no local memory)
        const uint32_t w = k < 4 ? hd.y : k < 8 ? hd.z : hd.w;
        return (w >> (8 * (k & 3))) & 0xFFu;
    };
    const int j = 2 * p + h;
    unsigned s_, m_;
    if (j < 4) s_ = sc(j) & 63, m_ = sc(j + 4) & 63;
    else s_ = (sc(j + 4) & 15) | ((sc(j - 4) >> 6) << 4), m_ = (sc(j + 4) >> 4) | ((sc(j) >> 6) << 4);
    const float a = d * (float)s_, b = dmin * (float)m_;
    const uint64_t a2 = dup2(a), mb2 = dup2(-b), nb2 = dup2(-8388608.0f);
    const uint4 *q4 = reinterpret_cast<const uint4 *>(blk + 16 + 32 * p);
#pragma unroll
    for (int half = 0; half < 2; half++) {  // 16 bytes -> weights 16*half .. +15 of the sub-block
        const uint4 qv = q4[half];
        const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
        {
            uint32_t out[8];
#pragma unroll
            for (int wd = 0; wd < 4; wd++) {
                const uint32_t v = h ? (qw[wd] >> 4) & 0x0F0F0F0Fu : qw[wd] & 0x0F0F0F0Fu;
                // a * q - b with one rounding (q * a is exact), two weights an instruction
                out[2 * wd] = pack16x2<F16>(fma_f32x2(codes2(v, SEL_B0, SEL_B1, nb2), a2, mb2));
                out[2 * wd + 1] = pack16x2<F16>(fma_f32x2(codes2(v, SEL_B2, SEL_B3, nb2), a2, mb2));
            }
            // columns 32*h + 16*half .. +15 = 16-byte chunks c0, c0 + 1 of the 128-byte row
            const int c0 = 4 * h + 2 * half;
#pragma unroll
            for (int cc = 0; cc < 2; cc++) {
                const int c = c0 + cc;
                *reinterpret_cast<uint4 *>(row + ((c ^ (r & 7)) << 4)) =
                    make_uint4(out[4 * cc], out[4 * cc + 1], out[4 * cc + 2], out[4 * cc + 3]);
            }
        }
    }
}

// Q4_K, both sub-blocks 2p (low nibbles: columns 0..31 of the stage) and 2p + 1 (high
// nibbles: 32..63) of byte pair p -- one load of the block head and of the 32 code bytes
// they share -- into the whole 128-byte swizzled row.
template <bool F16>
__device__ __forceinline__ void q4k_row_to_16(const uint8_t *blk, int p, uint8_t *row, int r)
{
    const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
    const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
    auto sc = [&](int k) {
        const uint32_t w = k < 4 ? hd.y : k < 8 ? hd.z : hd.w;
        return (w >> (8 * (k & 3))) & 0xFFu;
    };
    uint64_t a2[2], mb2[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int j = 2 * p + h;
        unsigned s_, m_;
        if (j < 4) s_ = sc(j) & 63, m_ = sc(j + 4) & 63;
        else s_ = (sc(j + 4) & 15) | ((sc(j - 4) >> 6) << 4), m_ = (sc(j + 4) >> 4) | ((sc(j) >> 6) << 4);
        a2[h] = dup2(d * (float)s_), mb2[h] = dup2(-(dmin * (float)m_));
    }
    const uint64_t nb2 = dup2(-8388608.0f);
    const uint4 *q4 = reinterpret_cast<const uint4 *>(blk + 16 + 32 * p);
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const uint4 qv = q4[half];
        const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
        for (int h = 0; h < 2; h++) {
            uint32_t out[8];
#pragma unroll
            for (int wd = 0; wd < 4; wd++) {
                const uint32_t v = h ? (qw[wd] >> 4) & 0x0F0F0F0Fu : qw[wd] & 0x0F0F0F0Fu;
                out[2 * wd] = pack16x2<F16>(fma_f32x2(codes2(v, SEL_B0, SEL_B1, nb2), a2[h], mb2[h]));
                out[2 * wd + 1] = pack16x2<F16>(fma_f32x2(codes2(v, SEL_B2, SEL_B3, nb2), a2[h], mb2[h]));
            }
            const int c0 = 4 * h + 2 * half;
#pragma unroll
            for (int cc = 0; cc < 2; cc++) {
                const int c = c0 + cc;
                *reinterpret_cast<uint4 *>(row + ((c ^ (r & 7)) << 4)) =
                    make_uint4(out[4 * cc], out[4 * cc + 1], out[4 * cc + 2], out[4 * cc + 3]);
            }
        }
    }
}

struct Args {
    int rows, cols, n;
    float *y;      // [n][rows]
    int kslices;   // > 1: CTA z takes K slice z (whole 256-column blocks) and writes part[z]
    float *part;   // [kslices][n][rows]
};

// Partial sums of the K slices -> Y, in slice order.
__global__ void pf_reduce_kernel(const float *__restrict__ part, float *__restrict__ y, long long total, int kslices)
{
    griddep_wait();
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        float v = part[i];
        for (int z = 1; z < kslices; z++) v += part[(long long)z * total + i];
        y[i] = v;
    }
}

constexpr int MAX_SPLIT_CTAS = 160;  // CTAs of a K-split launch at most (bounds the partials)
constexpr size_t PART_BYTES = (size_t)MAX_SPLIT_CTAS * BM * BN * 4;

template <bool F16>
__global__ void __launch_bounds__(THREADS, 1)
    pf_gemm_q4k_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, Args a)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const Smem s = carve(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * BM, tok0 = blockIdx.y * BN;
    const int KS = a.cols / BK / a.kslices;  // stages of this CTA's K slice
    const int ks0 = (int)blockIdx.z * KS;     // its first stage (a multiple of 4: whole blocks)
    if (threadIdx.x == 0) {
        for (int i = 0; i < NST; i++) {
            tcmv::mbar_init(&s.x_full[i], 1);
            tcmv::mbar_init(&s.w_full[i], NDQ);
            tcmv::mbar_init(&s.st_empty[i], 1);
        }
        for (int i = 0; i < NRAW; i++) {
            tcmv::mbar_init(&s.raw_full[i], 1);
            tcmv::mbar_init(&s.raw_empty[i], NDQ);
        }
        tcmv::mbar_init(s.acc_full, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         tcmv::smem_u32(s.tmem_addr)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *s.tmem_addr;
    griddep_wait();  // X (bf16) is written by the previous kernel
    bool failed = false;

    if (warp == 0) {
        if (lane == 0) {
            const uint64_t pol = tcmv::l2_evict_first();
            for (int ks = 0; ks < KS && !failed; ks++) {
                const int st = ks % NST;
                if (ks % 4 == 0) {  // a new raw block column
                    const int rk = ks / 4, rs = rk % NRAW;
                    if (rk >= NRAW && !tcmv::mbar_wait(&s.raw_empty[rs], ((rk / NRAW) - 1) & 1, WAIT)) {
                        failed = true;
                        break;
                    }
                    tcmv::mbar_expect_tx_arrive(&s.raw_full[rs], (unsigned)RAW_BYTES);
                    tcmv::tma_load_2d(s.raw(rs), &wmap, (rk + ks0 / 4) * (RAW_ROWB / 8), row0, &s.raw_full[rs], pol);
                }
                if (ks >= NST && !tcmv::mbar_wait(&s.st_empty[st], ((ks / NST) - 1) & 1, WAIT)) {
                    failed = true;
                    break;
                }
                tcmv::mbar_expect_tx_arrive(&s.x_full[st], (unsigned)X_BYTES);
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
                    "{%2, %3}], [%4];" ::"r"(tcmv::smem_u32(s.x(st))),
                    "l"(&xmap), "r"((ks0 + ks) * BK), "r"(tok0), "r"(tcmv::smem_u32(&s.x_full[st]))
                    : "memory");
            }
            if (failed) set_dev_error(0x71u);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int ks = 0; ks < KS; ks++) {
                const int st = ks % NST;
                const unsigned par = (ks / NST) & 1;
                if (!tcmv::mbar_wait(&s.x_full[st], par, WAIT) || !tcmv::mbar_wait(&s.w_full[st], par, WAIT)) {
                    failed = true;
                    set_dev_error(0x72u);
                    break;
                }
                fence_after_sync();
                const uint64_t ad = sw128_desc(s.w(st)), bd = sw128_desc(s.x(st));
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++)  // K16 slices: 32 bytes along the swizzled row
                    mma_16bit<F16>(tmem, ad + (uint64_t)(2 * kk), bd + (uint64_t)(2 * kk), (ks | kk) ? 1u : 0u);
                mma_commit(&s.st_empty[st]);
            }
            mma_commit(s.acc_full);  // completion of every MMA issued above (even after a failure)
        }
        __syncwarp();
    } else {
        // dequantisers: thread t takes weight row t % 128, nibble half t / 128
        const int r = (threadIdx.x - 64) & (BM - 1), hh = (threadIdx.x - 64) / BM;
        for (int ks = 0; ks < KS && !failed; ks++) {
            const int st = ks % NST, rk = ks / 4, rs = rk % NRAW, p = ks % 4;
            if (p == 0 && !tcmv::mbar_wait(&s.raw_full[rs], (rk / NRAW) & 1, WAIT)) failed = true;
            if (!failed && ks >= NST && !tcmv::mbar_wait(&s.st_empty[st], ((ks / NST) - 1) & 1, WAIT)) failed = true;
            if (failed) {
                set_dev_error(0x73u);
                break;
            }
            q4k_half_to_16<F16>(s.raw(rs) + r * RAW_ROWB, p, hh, s.w(st) + r * 128, r);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> MMA reads
            __syncwarp();
            if (lane == 0) {
                tcmv::mbar_arrive(&s.w_full[st]);
                if (p == 3) tcmv::mbar_arrive(&s.raw_empty[rs]);
            }
        }
        // epilogue: the accumulators of this warp's 32 lanes (rows)
        if (tcmv::mbar_wait(s.acc_full, 0, WAIT)) {
            fence_after_sync();
            const int q = warp & 3, row = row0 + 32 * q + lane;
            float *dst = a.kslices > 1 ? a.part + (size_t)blockIdx.z * a.n * a.rows : a.y;
            const int c0 = ((warp - 2) / 4) * (BN * 4 / NDQ);  // warps of one lane quadrant split the columns
            for (int c = c0; c < c0 + BN * 4 / NDQ; c += 32) {
                float v[32];
                tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c, v);
                if (row < a.rows) {
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const int tok = tok0 + c + i;
                        if (tok < a.n) dst[(size_t)tok * a.rows + row] = v[i];
                    }
                }
            }
        } else {
            set_dev_error(0x74u);
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
    griddep_launch();
}

// X f32 [n][cols] -> 16-bit operands (round to nearest even), 8 elements per thread.
template <bool F16>
__global__ void x_to_16_kernel(const float *__restrict__ x, uint16_t *__restrict__ xb, long long total8)
{
    griddep_wait();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < total8) {
        const float4 v0 = reinterpret_cast<const float4 *>(x)[2 * i], v1 = reinterpret_cast<const float4 *>(x)[2 * i + 1];
        reinterpret_cast<uint4 *>(xb)[i] = make_uint4(pack16<F16>(v0.x, v0.y), pack16<F16>(v0.z, v0.w),
                                                      pack16<F16>(v1.x, v1.y), pack16<F16>(v1.z, v1.w));
    }
    griddep_launch();
}

inline int make_x_map(CUtensorMap *m, const void *xb, int n, int cols, bool f16)
{
    tcmv::EncodeTiledFn fn = tcmv::encode_fn();
    if (!fn) return -6;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)n};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BN};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                    const_cast<void *>(xb), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -7;
}

inline int make_q4k_map(CUtensorMap *m, const void *w, int rows, int cols)
{
    tcmv::EncodeTiledFn fn = tcmv::encode_fn();
    if (!fn) return -6;
    const cuuint64_t rb = (cuuint64_t)(cols / 256) * 144;
    cuuint64_t dims[2] = {rb / 8, (cuuint64_t)rows};
    cuuint64_t strides[1] = {rb};
    cuuint32_t box[2] = {RAW_ROWB / 8, (cuuint32_t)BM};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(w), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -7;
}

}  // namespace pf
}  // namespace sb

namespace sb {
namespace pf {
template <bool F16>
int matmul(const void *w, size_t rows, size_t cols, size_t n, const float *x, float *y, void *ws, int pdl,
           cudaStream_t s)
{
    uint16_t *xb = reinterpret_cast<uint16_t *>(ws);
    const long long total8 = (long long)n * (long long)cols / 8;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((unsigned)((total8 + 255) / 256));
    c.blockDim = dim3(256);
    c.stream = s;
    c.attrs = at;
    c.numAttrs = pdl ? 1 : 0;
    if (cudaLaunchKernelEx(&c, x_to_16_kernel<F16>, x, xb, total8) != cudaSuccess) return -4;
    CUtensorMap wm, xm;
    int rc = make_q4k_map(&wm, w, (int)rows, (int)cols);
    if (!rc) rc = make_x_map(&xm, xb, (int)n, (int)cols, F16);
    if (rc) return rc;
    static size_t smem_rec[64];
    static std::mutex mu;
    {
        std::lock_guard<std::mutex> lk(mu);
        if ((rc = tcmv::ensure_smem(pf_gemm_q4k_kernel<F16>, smem_bytes(), smem_rec))) return rc;
    }
    // too few output tiles to fill the GPU: split K into slices of whole blocks (each CTA one
    // slice of one tile, partial sums reduced in slice order by a second launch)
    const int tiles = (int)(((rows + BM - 1) / BM) * ((n + BN - 1) / BN)), nblk = (int)(cols / 256);
    const int sms = num_sms_cached() < MAX_SPLIT_CTAS ? num_sms_cached() : MAX_SPLIT_CTAS;
    int ksl = 1;
    // (not for K of one or two blocks: there the extra reduction launch costs more than it saves)
    while (nblk >= 4 && 2 * ksl <= nblk && nblk % (2 * ksl) == 0 && tiles * 2 * ksl <= sms) ksl *= 2;
    float *part = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + ((n * cols * 2 + 255) & ~(size_t)255));
    Args a{(int)rows, (int)cols, (int)n, y, ksl, part};
    c.gridDim = dim3((unsigned)((rows + BM - 1) / BM), (unsigned)((n + BN - 1) / BN), (unsigned)ksl);
    c.blockDim = dim3(THREADS);
    c.dynamicSmemBytes = smem_bytes();
    c.numAttrs = 1;  // X comes from the conversion just launched
    if (cudaLaunchKernelEx(&c, pf_gemm_q4k_kernel<F16>, wm, xm, a) != cudaSuccess) return -4;
    if (ksl == 1) return 0;
    const long long total = (long long)n * (long long)rows;
    c.gridDim = dim3((unsigned)(((total + 255) / 256) < 1184 ? (total + 255) / 256 : 1184));
    c.blockDim = dim3(256);
    c.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&c, pf_reduce_kernel, (const float *)part, y, total, ksl) == cudaSuccess ? 0 : -4;
}
}  // namespace pf
}  // namespace sb

extern "C" size_t sbk_matmul_ws_bytes(size_t n, size_t cols)
{
    // X as 16-bit operands, then the partial sums of a K-split launch (bounded by its CTAs)
    return ((n * cols * 2 + 255) & ~(size_t)255) + sb::pf::PART_BYTES + 256;
}

extern "C" int sbk_matmul(uint8_t dtype, const void *w, size_t rows, size_t cols, size_t n, const float *x, float *y,
                          void *ws, int prec, int pdl, void *stream)
{
    if (!w || !x || !y || !ws || !rows || !n || !cols) return -1;
    if (dtype != SB_DTYPE_Q4_K) return -5;
    if (prec != SBK_PREC_BF16 && prec != SBK_PREC_F16) return -1;
    if (cols % 256 || cols > (1u << 20) || rows > (1u << 24) || n > (1u << 24)) return -1;
    if (((uintptr_t)w | (uintptr_t)x | (uintptr_t)ws) & 15) return -2;
    return prec == SBK_PREC_F16 ? sb::pf::matmul<true>(w, rows, cols, n, x, y, ws, pdl, (cudaStream_t)stream)
                                : sb::pf::matmul<false>(w, rows, cols, n, x, y, ws, pdl, (cudaStream_t)stream);
}
