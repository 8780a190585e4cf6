// tc_q80.cuh -- the .som Q8_0 format of the tensor-core matvec (tc_mmv.cuh).
//
// .som Q8_0 (crates/sosomodel/src/layout.rs:57-59, dequant.rs:74-102): blocks of 32
// weights, an f32 scale then 32 int8 codes (36 bytes); gemm::matvec_q8_0
// (crates/soso-llm-core/src/gemm.rs:295-332) forms per block scale * sum(q * x).
//
// The framework's unit here is 128 weights (four blocks, 144 bytes of a row), so stages
// are 16 rows x 4 units (576 bytes of a row, boxes 16 bytes wider) as for Q4_K.  TMA needs rows that start
// 16-byte aligned: a row of cols/32 blocks is a multiple of 16 bytes when cols is a
// multiple of 128; other widths (10944) are held with their rows padded to 16 bytes
// (SB_DTYPE_Q8_0_R, made on upload by sbk_q80_pad), same blocks, same bytes.
//
// Numerics.  The codes enter an s8 x s8 -> s32 MMA (m16n8k32: one block of 16 rows per
// MMA) straight from shared memory; x enters as four int8 pieces per element (as for
// Q4_K, 28 significant bits, one exponent per 128 elements), pieces 0..3 in B columns
// 0..3 (columns 4..7 zero).  The integer block dots are exact; each is scaled by the
// block's f32 scale in f32, as the reference does per block.
#pragma once
#include "tc_common.cuh"

namespace sb {
namespace tcmv {

// Row bytes of a Q8_0 row as the tensor-core kernel reads it: padded to 16 bytes.
__host__ __device__ inline size_t q80_row_bytes_padded(size_t cols) { return ((cols / 32) * 36 + 15) & ~(size_t)15; }

// Copy Q8_0 rows (reference layout, device memory) to 16-byte-aligned rows, zero padding.
__global__ void q80_pad_kernel(const uint8_t *__restrict__ src, long long rows, int rb, uint8_t *__restrict__ dst,
                               int rbp)
{
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * rbp) return;
    const long long r = i / rbp;
    const int o = (int)(i - r * rbp);
    dst[i] = o < rb ? src[r * rb + o] : 0;
}

#ifndef SB_Q80_NSTREAM
#define SB_Q80_NSTREAM 3  // consumer teams (build-time tuning knob)
#endif
#ifndef SB_Q80_NSLOT
#define SB_Q80_NSLOT 9  // ring slots, a multiple of the teams (build-time tuning knob)
#endif
#ifndef SB_Q80_MINB
#define SB_Q80_MINB 1  // CTAs per SM the kernels are compiled for (build-time tuning knob)
#endif

struct Q80 {
    static constexpr uint8_t DTYPE = 15;  // SB_DTYPE_Q8_0_R (also reads SB_DTYPE_Q8_0 rows whose width is a multiple of 128)
    static constexpr int SBLK = 4;        // units (4 blocks, 128 weights) per stage
    static constexpr int NCONS = 4;
    static constexpr int NSTREAM = SB_Q80_NSTREAM;
    static constexpr int NCW = NCONS * NSTREAM;
    static constexpr int THREADS = (NCW + 1) * 32;
    static constexpr int MINB = SB_Q80_MINB;
    static constexpr int NSLOT = SB_Q80_NSLOT;  // a multiple of NSTREAM
    static constexpr int BOXW = SBLK * 18 + 2;  // u64 per box row: one stage (576 B) + 16 B, so that
                                                // rows are 148 words apart and the 4-byte fragment loads
                                                // of a warp hit 32 distinct banks
    static constexpr int ROWB = BOXW * 8;
    static constexpr int SLOTB = 16 * ROWB;
    static constexpr int MAX_COLS = 16384;
    static constexpr int UNIT = 128;      // weights per framework unit
    static constexpr int COLS_MULT = 32;  // whole blocks

    __host__ __device__ static size_t row_bytes(int cols) { return q80_row_bytes_padded((size_t)cols); }
    __host__ __device__ static int stage_x(int j) { return j * SBLK * 18; }
    __host__ __device__ static int units(int cols) { return (cols + UNIT - 1) / UNIT; }

    // Prepared x per unit u of 128 elements: frag [u][4 blocks][4 pieces][8 quads] u32 (512 B),
    // then fx [u] f32 = 2^(ex - 7), the weight of piece 0.
    __host__ __device__ static size_t prep_bytes(int cols) { return ((size_t)units(cols) * 516 + 15) & ~(size_t)15; }

    // Lane l holds elements 4l..4l+3 of the unit (v[0], zero past the row's end): block l/8, quad l%8.
    static constexpr int XPL = 1;
    __device__ static int xidx(int u, int l, int) { return u * 32 + l; }
    __device__ static void prep_unit(int u, int nu, const float4 (&vx)[XPL], uint8_t *prep)
    {
        const int l = threadIdx.x & 31;
        uint32_t *frag = reinterpret_cast<uint32_t *>(prep);
        float *fx = reinterpret_cast<float *>(prep + (size_t)nu * 512);
        {
            const float4 v = vx[0];
            const float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
            const int ex = warp_exp_above(mx);
            const float scl = pow2f(7 - ex);
            uint32_t pk[4];
            int8_pieces4(make_float4(v.x * scl, v.y * scl, v.z * scl, v.w * scl), pk);
            const int b = l >> 3, q = l & 7;
#pragma unroll
            for (int pc = 0; pc < 4; pc++) frag[((u * 4 + b) * 4 + pc) * 8 + q] = pk[pc];
            if (l == 0) fx[u] = pow2f(ex - 7);
        }
    }

    struct Lane {
        int g, t;
        bool live;
        float lanefac;
    };
    __device__ static Lane lane_setup(int g, int t)
    {
        Lane L;
        L.g = g, L.t = t;
        L.live = g < 4;                              // B columns 0..3 carry pieces 0..3
        L.lanefac = t == 1 ? 1.0f / 16384.0f : 1.0f;  // D columns (2t, 2t+1): pieces 2t, 2t+1
        return L;
    }

    struct Seg {
        const uint32_t *bfl;  // this lane's piece row of unit 0, block 0
        int bu, bk;           // u32 strides per unit / per block (0 for lanes without x)
        const float *fxp;
        int nb32;             // blocks per row
    };
    __device__ static Seg seg_setup(const Lane &L, const uint8_t *prep, const uint8_t *zero, int nb, int cols)
    {
        Seg s;
        s.bfl = L.live ? reinterpret_cast<const uint32_t *>(prep) + L.g * 8 + L.t
                       : reinterpret_cast<const uint32_t *>(zero);
        s.bu = L.live ? 128 : 0;
        s.bk = L.live ? 32 : 0;
        s.fxp = reinterpret_cast<const float *>(prep + (size_t)nb * 512);
        s.nb32 = cols / 32;
        return s;
    }

    // Unit `blk` (4 blocks) of the stage in `slot`: copy this warp's bytes to registers,
    // release the slot, accumulate.  nb = units per row.
    __device__ static void block(const Lane &L, const Seg &S, const uint8_t *slot, int cw, int blk, int nb,
                                 uint64_t *empty, float &acc0, float &acc1)
    {
        const int lane = threadIdx.x & 31;
        const uint8_t *r0p = slot + L.g * ROWB + cw * 144, *r1p = r0p + 8 * ROWB;
        uint32_t a[4][4];
        float d0[4], d1[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint8_t *b0 = r0p + 36 * k, *b1 = r1p + 36 * k;
            d0[k] = *reinterpret_cast<const float *>(b0);
            d1[k] = *reinterpret_cast<const float *>(b1);
            a[k][0] = *reinterpret_cast<const uint32_t *>(b0 + 4 + 4 * L.t);
            a[k][1] = *reinterpret_cast<const uint32_t *>(b1 + 4 + 4 * L.t);
            a[k][2] = *reinterpret_cast<const uint32_t *>(b0 + 20 + 4 * L.t);
            a[k][3] = *reinterpret_cast<const uint32_t *>(b1 + 20 + 4 * L.t);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty);
        const int nb32 = S.nb32;
        const float fx = S.fxp[blk] * L.lanefac;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            if (blk * 4 + k >= nb32) break;  // past the row's last block (zero-filled: skip)
            const uint32_t *bp = S.bfl + (size_t)blk * S.bu + k * S.bk;
            int D[4] = {0, 0, 0, 0};
            mma_s8s8(D, a[k][0], a[k][1], a[k][2], a[k][3], bp[0], bp[4]);
            acc0 += (d0[k] * fx) * fmaf(__int2float_rn(D[1]), 1.0f / 128.0f, __int2float_rn(D[0]));
            acc1 += (d1[k] * fx) * fmaf(__int2float_rn(D[3]), 1.0f / 128.0f, __int2float_rn(D[2]));
        }
    }
};

}  // namespace tcmv
}  // namespace sb
