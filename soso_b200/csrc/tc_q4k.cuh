// tc_q4k.cuh -- the Q4_K format of the tensor-core matvec (tc_mmv.cuh).
//
// Same block layout and per-sub-block algebra as the reference
// (crates/sosomodel/src/dequant.rs:150-191; gemm.rs:428-461):
//   y[r] = sum_blocks ( d * sum_j sc_j * Sum_l q_l x_l  -  dmin * sum_j m_j * Sum_l x_l )
//
// Numerics.  The 4-bit codes enter a u8 x s8 -> s32 MMA (m16n8k32) as bytes:
// one AND of a qs word gives four low-nibble codes, another four high-nibble
// codes times 16 (not shifted; the 16 is folded into the scales).  x enters as
// four int8 pieces per element, x * 2^(7-ex) = p0 + p1/2^7 + p2/2^14 + p3/2^21
// with 2^ex above the block's max |x| (x * 2^(7-ex) rounded once to a multiple of
// 2^-21, then split into exact integer fields), one piece per B column.  Products and their sums are exact
// integers; the 6-bit scales multiply them in integer arithmetic (IMAD), and
// only the per-block result is converted to f32 and scaled by d.  The min term
// sum_j m_j * Sum x_j is one f16 MMA per block: m as f16 subnormals (exact)
// against the sub-block sums of x split into hi/lo f16 halves.  So the only
// rounding is f32 rounding of a few per-block terms and of the row sum.
//
// Fragment layout.  A lane (g = lane/4, t = lane%4) holds rows g and g+8 and,
// of byte pair P = 2*duo + t/2 of the block, bytes 16*(t%2)..+15.  Its k-slots
// of an MMA are thus all in one sub-block (2P for low nibbles, 2P+1 for high);
// B column g carries piece g%4 of x for sub-block slot g/4 and is zero where a
// lane's k-slots belong to the other slot, so D column pair (2t, 2t+1) holds
// pieces 2(t%2), 2(t%2)+1 of sub-block 2*(2*duo + t/2) + nib.  Eight MMAs per
// 16-row x 256-column tile, four independent accumulators of two each.
//
// Stage: 16 rows x 4 blocks (a 576-byte box row; 576 == 64 mod 128, so the
// fragment loads are bank-conflict-free); 12 consumer warps in 3 teams of 4,
// one block per warp per stage.
#pragma once
#ifndef SB_Q4K_NSLOT
#define SB_Q4K_NSLOT 9  // ring slots (build-time tuning knob)
#endif
#ifndef SB_Q4K_NSTREAM
#define SB_Q4K_NSTREAM 3  // consumer teams (build-time tuning knob)
#endif
#ifndef SB_Q4K_MINB
#define SB_Q4K_MINB 1  // CTAs per SM the engine's matvec is compiled for (build-time tuning knob)
#endif
#include "tc_common.cuh"

namespace sb {
namespace tcmv {

struct Q4K {
    static constexpr uint8_t DTYPE = 3;  // SB_DTYPE_Q4_K
    static constexpr int SBLK = 4;       // blocks per stage
    static constexpr int NCONS = 4;      // consumer warps per stage (one block each)
    static constexpr int NSTREAM = SB_Q4K_NSTREAM;  // stages in compute at once (teams)
    static constexpr int NCW = NCONS * NSTREAM;
    static constexpr int THREADS = (NCW + 1) * 32;
    static constexpr int MINB = SB_Q4K_MINB;
    static constexpr int NSLOT = SB_Q4K_NSLOT;  // a multiple of NSTREAM
    static constexpr int BOXW = SBLK * 18;  // u64 per box row (576 B)
    static constexpr int ROWB = BOXW * 8;
    static constexpr int SLOTB = 16 * ROWB;
    static constexpr int MAX_COLS = 16384;

    static constexpr int COLS_MULT = 256;
    __host__ __device__ static int units(int cols) { return cols / 256; }
    __host__ __device__ static size_t row_bytes(int cols) { return (size_t)(cols / 256) * 144; }
    __host__ __device__ static int stage_x(int j) { return j * SBLK * 18; }  // u64 column of stage j

    // Prepared x, per CTA in shared memory, per block b of 256 elements:
    //   frag [nb][4 q][16 live lanes][4] u32 -- int8 x pieces in B-fragment order
    //   mfr  [nb][2 g][4 t] u32 -- f16x2 sub-block sums of x, hi (g = 0) / lo (g = 1):
    //        the B fragment of the MMA that forms the min terms
    //   fx   [nb] f32 -- 2^(ex - 11): weight of piece 0 (and the 1/16 of the high nibbles)
    //   fm   [nb] f32 -- 2^(9 + kx): undoes the scaling of the min-term MMA
    // (rounded to 16 B: the zero area read as uint4 follows it)
    __host__ __device__ static size_t prep_bytes(int cols)
    {
        return ((size_t)(cols / 256) * (1024 + 32 + 8) + 15) & ~(size_t)15;
    }

    // x -> prep, one block b (unit) per warp at a time; lane l holds elements 4l..4l+3
    // (v[0]) and 128+4l..128+4l+3 (v[1]).  Element e of sub-block s, piece p, goes to
    // live lane L = 2(4*((s>>1)&1) + p) + (e>>4), register
    // 4*(2*(s>>2) + (s&1)) + 2*((e>>3)&1) + ((e>>2)&1), byte e&3.
    static constexpr int XPL = 2;  // float4 of x per lane per unit
    __device__ static int xidx(int b, int l, int k) { return b * 64 + 32 * k + l; }
    __device__ static void prep_unit(int b, int nb, const float4 (&v)[XPL], uint8_t *prep)
    {
        const int l = threadIdx.x & 31;
        uint32_t *frag = reinterpret_cast<uint32_t *>(prep);
        unsigned short *mfr = reinterpret_cast<unsigned short *>(prep + (size_t)nb * 1024);
        float *fx = reinterpret_cast<float *>(prep + (size_t)nb * 1056), *fm = fx + nb;
        {
            const float4 va = v[0], vb = v[1];
            const float mx = fmaxf(fmaxf(fmaxf(fabsf(va.x), fabsf(va.y)), fmaxf(fabsf(va.z), fabsf(va.w))),
                                   fmaxf(fmaxf(fabsf(vb.x), fabsf(vb.y)), fmaxf(fabsf(vb.z), fabsf(vb.w))));
            float sa = (va.x + va.y) + (va.z + va.w), sbv = (vb.x + vb.y) + (vb.z + vb.w);
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                sa += __shfl_xor_sync(0xffffffffu, sa, o);
                sbv += __shfl_xor_sync(0xffffffffu, sbv, o);
            }
            const int ex = warp_exp_above(mx);
            const float scl = pow2f(7 - ex);
            auto pieces = [&](float4 v4, int n) {
                const int sblk = n >> 5, e = n & 31;
                const int sig = (sblk >> 1) & 1, q = 2 * (sblk >> 2) + (sblk & 1);
                const int word = 2 * ((e >> 3) & 1) + ((e >> 2) & 1), tp = e >> 4;
                uint32_t pk[4];
                int8_pieces4(make_float4(v4.x * scl, v4.y * scl, v4.z * scl, v4.w * scl), pk);
#pragma unroll
                for (int pc = 0; pc < 4; pc++) {
                    const int L = 2 * (4 * sig + pc) + tp;
                    frag[((b * 4 + q) * 16 + L) * 4 + word] = pk[pc];
                }
            };
            pieces(va, 4 * l);
            pieces(vb, 128 + 4 * l);
            // sub-block sums -> f16 hi/lo with one power-of-two scale per block (max below 2^15)
            const int kx = warp_exp_above(fmaxf(fabsf(sa), fabsf(sbv)));
            const float ms = pow2f(15 - kx);
            if ((l & 7) == 0) {
                const float sv[2] = {sa, sbv};
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const int sidx = 4 * c + (l >> 3);
                    const float sm = sv[c] * ms;
                    const __half hi = __float2half_rn(sm), lo = __float2half_rn(sm - __half2float(hi));
                    mfr[((b * 2 + 0) * 4 + (sidx >> 1)) * 2 + (sidx & 1)] = __half_as_ushort(hi);
                    mfr[((b * 2 + 1) * 4 + (sidx >> 1)) * 2 + (sidx & 1)] = __half_as_ushort(lo);
                }
            }
            if (l == 0) {
                fx[b] = pow2f(ex - 11);
                fm[b] = pow2f(9 + kx);
            }
        }
    }

    // Per-lane constants.
    struct Lane {
        int g, t, q2, qoff, sc_sh;
        bool live, mlive;
        uint32_t sel_m;
        float lanefac;
    };
    __device__ static Lane lane_setup(int g, int t)
    {
        Lane L;
        L.g = g, L.t = t, L.q2 = t >> 1;
        // B columns are (sub-block slot g/4, piece g%4): a lane carries x only where
        // its k-slots (sub-block slot t/2) meet its column
        L.live = (g >> 2) == L.q2, L.mlive = g < 2;
        L.qoff = 16 + t * 16;  // + 64 * duo
        L.sc_sh = 16 * L.q2;
        // min-term A fragment: m of sub-blocks 2t, 2t+1 as f16 subnormals (byte -> u16 lane)
        L.sel_m = (uint32_t)((2 * t) & 3) | 0x40u | ((uint32_t)(((2 * t) & 3) + 1) << 8) | 0x4000u;
        L.lanefac = (t & 1) ? 1.0f / 16384.0f : 1.0f;  // pieces 2, 3 weigh 2^-14 of pieces 0, 1
        return L;
    }

    // Pointers into the prepared x of one matrix.
    struct Seg {
        const uint4 *bfl;
        int bq, bb;
        const uint32_t *mfl;
        int mb;
        const float *fxp, *fmp;
    };
    __device__ static Seg seg_setup(const Lane &L, const uint8_t *prep, const uint8_t *zero, int nb, int)
    {
        Seg s;
        // lanes without x read zeros: stride 0 into the zero area
        s.bfl = L.live ? reinterpret_cast<const uint4 *>(prep) + 2 * L.g + (L.t & 1)
                       : reinterpret_cast<const uint4 *>(zero);
        s.bq = L.live ? 16 : 0, s.bb = L.live ? 64 : 0;
        s.mfl = L.mlive ? reinterpret_cast<const uint32_t *>(prep + (size_t)nb * 1024) + L.g * 4 + L.t
                        : reinterpret_cast<const uint32_t *>(zero);
        s.mb = L.mlive ? 8 : 0;
        s.fxp = reinterpret_cast<const float *>(prep + (size_t)nb * 1056);
        s.fmp = s.fxp + nb;
        return s;
    }

    // Block `blk` of the stage in `slot` (rows g and g+8 at r0p, r1p): copy this
    // warp's bytes to registers, release the slot, accumulate into acc0 / acc1.
    __device__ static void block(const Lane &L, const Seg &S, const uint8_t *slot, int cw, int blk, int nb,
                                 uint64_t *empty, float &acc0, float &acc1)
    {
        const int lane = threadIdx.x & 31;
        const uint8_t *r0p = slot + L.g * ROWB + cw * 144, *r1p = r0p + 8 * ROWB;
        const uint4 h0 = *reinterpret_cast<const uint4 *>(r0p);
        const uint4 h1 = *reinterpret_cast<const uint4 *>(r1p);
        // rows g / g+8: 16 bytes of pair 2*duo + t/2 each (bytes 16*(t&1).. of the pair)
        const uint4 qa0 = *reinterpret_cast<const uint4 *>(r0p + L.qoff);
        const uint4 qa1 = *reinterpret_cast<const uint4 *>(r0p + L.qoff + 64);
        const uint4 qb0 = *reinterpret_cast<const uint4 *>(r1p + L.qoff);
        const uint4 qb1 = *reinterpret_cast<const uint4 *>(r1p + L.qoff + 64);
        // The stage's bytes are in registers: hand the slot back to the producer
        // now (arrive has release semantics, so these reads precede its refill).
        __syncwarp();
        if (lane == 0) mbar_arrive(empty);
        const uint4 *bp = S.bfl + blk * S.bb;
        const uint4 B0 = bp[0], B1 = bp[S.bq], B2 = bp[2 * S.bq], B3 = bp[3 * S.bq];
        const uint32_t mbv = S.mfl[blk * S.mb];
        // D[2*duo + nib]: sub-block 2*(2*duo + t/2) + nib; columns (2t, 2t+1) = pieces
        // 2(t&1), 2(t&1)+1; rows g (c0, c1) and g+8 (c2, c3).  Integer, exact.
        constexpr uint32_t LO = 0x0F0F0F0Fu, HI = 0xF0F0F0F0u;
        int D[4][4];
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
            for (int c = 0; c < 4; c++) D[a][c] = 0;
        mma_u8s8(D[0], qa0.x & LO, qb0.x & LO, qa0.y & LO, qb0.y & LO, B0.x, B0.y);
        mma_u8s8(D[1], qa0.x & HI, qb0.x & HI, qa0.y & HI, qb0.y & HI, B1.x, B1.y);
        mma_u8s8(D[2], qa1.x & LO, qb1.x & LO, qa1.y & LO, qb1.y & LO, B2.x, B2.y);
        mma_u8s8(D[3], qa1.x & HI, qb1.x & HI, qa1.y & HI, qb1.y & HI, B3.x, B3.y);
        mma_u8s8(D[0], qa0.z & LO, qb0.z & LO, qa0.w & LO, qb0.w & LO, B0.z, B0.w);
        mma_u8s8(D[1], qa0.z & HI, qb0.z & HI, qa0.w & HI, qb0.w & HI, B1.z, B1.w);
        mma_u8s8(D[2], qa1.z & LO, qb1.z & LO, qa1.w & LO, qb1.w & LO, B2.z, B2.w);
        mma_u8s8(D[3], qa1.z & HI, qb1.z & HI, qa1.w & HI, qb1.w & HI, B3.z, B3.w);
        // 6-bit scales and mins (dequant.rs:150-167 packing), rows g and g+8
        auto sc_pack = [&](const uint4 h, int (&c)[4], uint32_t &am) {
            const uint32_t S0 = h.y & 0x3F3F3F3Fu;
            const uint32_t S1 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
            const uint32_t M0 = h.z & 0x3F3F3F3Fu;
            const uint32_t M1 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
            const uint32_t s0 = S0 >> L.sc_sh, s1 = S1 >> L.sc_sh;
            // low-nibble sub-blocks carry codes x1, high-nibble ones x16: scale the former by 16
            c[0] = (int)((s0 << 4) & 0xFF0u);
            c[1] = (int)((s0 >> 8) & 0xFFu);
            c[2] = (int)((s1 << 4) & 0xFF0u);
            c[3] = (int)((s1 >> 8) & 0xFFu);
            am = __byte_perm(L.t < 2 ? M0 : M1, 0u, L.sel_m);
        };
        int c0[4], c1[4];
        uint32_t am0, am1;
        sc_pack(h0, c0, am0);
        sc_pack(h1, c1, am1);
        // min terms: sum_j m_j * sumx_j for rows g, g+8 (column pair 0/1 = hi/lo, lane t = 0)
        float dm[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma_f16(dm, am0, am1, 0u, 0u, mbv, 0u);
        const int I00 = c0[0] * D[0][0] + c0[1] * D[1][0] + c0[2] * D[2][0] + c0[3] * D[3][0];
        const int I01 = c0[0] * D[0][1] + c0[1] * D[1][1] + c0[2] * D[2][1] + c0[3] * D[3][1];
        const int I10 = c1[0] * D[0][2] + c1[1] * D[1][2] + c1[2] * D[2][2] + c1[3] * D[3][2];
        const int I11 = c1[0] * D[0][3] + c1[1] * D[1][3] + c1[2] * D[2][3] + c1[3] * D[3][3];
        const float2 dn0 = __half22float2(*reinterpret_cast<const __half2 *>(&h0.x));
        const float2 dn1 = __half22float2(*reinterpret_cast<const __half2 *>(&h1.x));
        const float fxl = S.fxp[blk] * L.lanefac, fml = S.fmp[blk];
        acc0 += (dn0.x * fxl) * fmaf(__int2float_rn(I01), 1.0f / 128.0f, __int2float_rn(I00)) -
                (dn0.y * fml) * (dm[0] + dm[1]);
        acc1 += (dn1.x * fxl) * fmaf(__int2float_rn(I11), 1.0f / 128.0f, __int2float_rn(I10)) -
                (dn1.y * fml) * (dm[2] + dm[3]);
    }
};

}  // namespace tcmv
}  // namespace sb
