// tc_q6k.cuh -- the Q6_K format of the tensor-core matvec (tc_mmv.cuh), on a
// device-side repacking of the GGML Q6_K blocks.
//
// GGML Q6_K (crates/gguf2som/src/lib.rs:1639-1661): 256 weights in 210 bytes,
// ql[128] (low 4 bits), qh[64] (high 2 bits), 16 int8 scales, f16 d; in half n
// (128 weights), weight 32k + l (k = 0..3, l = 0..31) has
//   code = ((ql[64n + l + 32(k&1)] >> 4(k>>1)) & 15) | (((qh[32n + l] >> 2k) & 3) << 4)
//   w = d * sc[8n + 2k + l/16] * (code - 32).
// A 210-byte block puts its fields at 2-byte alignment and a row of 43 blocks
// (11008 columns) at a 9030-byte stride, which neither TMA (16-byte strides)
// nor vector loads accept.  So weights are repacked once, on upload, into
// groups of 8 blocks laid out as planes -- [ql 8x128][qh 8x64][sc 8x16][d 8x2]
// = 1680 bytes, no padding -- with a last group of m < 8 blocks laid out the
// same way with m and padded to 16 bytes.  Same bytes, same arithmetic.
//
// Numerics.  Codes (0..63, built with two masks and a shift per four codes)
// enter a u8 x s8 MMA (m16n8k32) against x as four int8 pieces (as for Q4_K);
// the int8 scales multiply the exact integer sums (IMAD); the -32 offset,
// -32 * sum_s sc_s * Sum_{l in s} x_l, is one s8 x s8 MMA per block: the scales
// (one word per lane, loaded as they lie) against the sub-block sums of the x
// pieces, split into two base-64 digits so they fit int8 (exact).
//
// Fragment layout.  One MMA per (half n, k): 32 weights = sub-blocks 2k (l <
// 16) and 2k+1 (l >= 16) of that half, for rows g and g+8.  Lane (g, t) takes
// l = 8t..8t+7, so its k-slots are all in sub-block slot t/2; B column g holds
// piece g%4 for slot g/4, as for Q4_K.  Stage: 16 rows x one group (8 blocks);
// 16 consumer warps in 2 teams of 8, one block per warp per stage.  The box
// row is 1696 bytes (one group + 16, == 32 mod 128: conflict-free 8-byte loads).
#pragma once
#ifndef SB_Q6K_NSLOT
#define SB_Q6K_NSLOT 4  // ring slots (build-time tuning knob)
#endif
#ifndef SB_Q6K_NSTREAM
#define SB_Q6K_NSTREAM 2  // consumer teams (build-time tuning knob)
#endif
#include "tc_common.cuh"

namespace sb {
namespace tcmv {

// Bytes of a packed Q6_K row of `cols` weights (cols a multiple of 256).
__host__ __device__ inline size_t q6k_packed_row_bytes(size_t cols)
{
    const size_t nb = cols / 256, full = nb / 8, m = nb % 8;
    return full * 1680 + (m ? (210 * m + 15) / 16 * 16 : 0);
}

// One thread per (row, block): GGML block -> its place in the row's group planes.
__global__ void q6k_pack_kernel(const uint8_t *__restrict__ src, long long rows, int nb, uint8_t *__restrict__ dst,
                                long long rbp)
{
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * nb) return;
    const long long r = i / nb;
    const int b = (int)(i - r * nb), gi = b / 8, w = b % 8, m = min(8, nb - 8 * gi);
    const uint8_t *s = src + i * 210;
    uint8_t *base = dst + r * rbp + (long long)gi * 1680;
    for (int k = 0; k < 128; k++) base[128 * w + k] = s[k];
    for (int k = 0; k < 64; k++) base[128 * m + 64 * w + k] = s[128 + k];
    for (int k = 0; k < 16; k++) base[192 * m + 16 * w + k] = s[192 + k];
    base[208 * m + 2 * w] = s[208];
    base[208 * m + 2 * w + 1] = s[209];
    if (m < 8 && w == m - 1)  // zero the padding of a last, partial group
        for (long long k = 210 * m; k < rbp - (long long)gi * 1680; k++) base[k] = 0;
}

struct Q6KP {
    static constexpr uint8_t DTYPE = 14;  // SB_DTYPE_Q6_K_P
    static constexpr int SBLK = 8;        // blocks per stage (one group)
    static constexpr int NCONS = 8;
    static constexpr int NSTREAM = SB_Q6K_NSTREAM;
    static constexpr int NCW = NCONS * NSTREAM;
    static constexpr int THREADS = (NCW + 1) * 32;
    static constexpr int MINB = 1;
    static constexpr int NSLOT = SB_Q6K_NSLOT;  // a multiple of NSTREAM
    static constexpr int BOXW = 212;  // u64: one group (210) + 16 bytes
    static constexpr int ROWB = BOXW * 8;
    static constexpr int SLOTB = 16 * ROWB;
    static constexpr int MAX_COLS = 12288;

    static constexpr int COLS_MULT = 256;
    __host__ __device__ static int units(int cols) { return cols / 256; }
    __host__ __device__ static size_t row_bytes(int cols) { return q6k_packed_row_bytes((size_t)cols); }
    __host__ __device__ static int stage_x(int j) { return j * 210; }

    // Prepared x per block b: frag [nb][4 q][16 live lanes][4] u32 (int8 pieces, B-fragment
    // order); ofr [nb][32 lanes] u32 (base-64 digits of the per-sub-block sums of the pieces,
    // B fragment of the offset MMA); fx [nb] f32 = 2^(ex - 7), the weight of piece 0.
    __host__ __device__ static size_t prep_bytes(int cols)
    {
        return ((size_t)(cols / 256) * (1024 + 128 + 4) + 15) & ~(size_t)15;
    }

    // Lane l holds elements 8l..8l+7 of the block: half n = l/16, k = (l/4)%4,
    // t = l%4 (l = 8t.. of the 32), so its pieces go to live lane 2(4*(t/2) + p) +
    // (t%2), register 4*((4n + k)/2) + 2*((4n + k)&1) + (4-element half), byte.
    static constexpr int XPL = 2;  // float4 of x per lane per unit: v[0] = elements 8l..8l+3, v[1] = 8l+4..8l+7
    __device__ static int xidx(int b, int l, int k) { return b * 64 + 2 * l + k; }
    __device__ static void prep_unit(int b, int nb, const float4 (&v)[XPL], uint8_t *prep)
    {
        const int l = threadIdx.x & 31;
        uint32_t *frag = reinterpret_cast<uint32_t *>(prep);
        int8_t *ofr = reinterpret_cast<int8_t *>(prep + (size_t)nb * 1024);
        float *fx = reinterpret_cast<float *>(prep + (size_t)nb * 1152);
        const int n = l >> 4, kk = (l >> 2) & 3, te = l & 3, sig = te >> 1, tp = te & 1;
        const int mi = 4 * n + kk, q = mi >> 1;
        {
            const float4 va = v[0], vb = v[1];
            const float mx = fmaxf(fmaxf(fmaxf(fabsf(va.x), fabsf(va.y)), fmaxf(fabsf(va.z), fabsf(va.w))),
                                   fmaxf(fmaxf(fabsf(vb.x), fabsf(vb.y)), fmaxf(fabsf(vb.z), fabsf(vb.w))));
            const int ex = warp_exp_above(mx);
            const float scl = pow2f(7 - ex);
            int sx[4] = {0, 0, 0, 0};
#pragma unroll
            for (int bsel = 0; bsel < 2; bsel++) {
                const float4 v4 = bsel ? vb : va;
                uint32_t pk[4];
                int8_pieces4(make_float4(v4.x * scl, v4.y * scl, v4.z * scl, v4.w * scl), pk);
                const int word = 2 * (mi & 1) + bsel;
#pragma unroll
                for (int pc = 0; pc < 4; pc++) {
                    frag[((b * 4 + q) * 16 + 2 * (4 * sig + pc) + tp) * 4 + word] = pk[pc];
#pragma unroll
                    for (int i = 0; i < 4; i++) sx[pc] += (int)(int8_t)((pk[pc] >> (8 * i)) & 0xFFu);
                }
            }
            // sub-block l/2 (16 elements) is held by lanes l and l^1
#pragma unroll
            for (int pc = 0; pc < 4; pc++) sx[pc] += __shfl_xor_sync(0xffffffffu, sx[pc], 1);
            if ((l & 1) == 0) {
                const int s = l >> 1;
#pragma unroll
                for (int pc = 0; pc < 4; pc++) {
                    const int hi = sx[pc] >> 6, lo = sx[pc] & 63;  // sx = 64 hi + lo, |sx| <= 2048
                    ofr[(b * 32 + (2 * pc) * 4 + (s >> 2)) * 4 + (s & 3)] = (int8_t)hi;
                    ofr[(b * 32 + (2 * pc + 1) * 4 + (s >> 2)) * 4 + (s & 3)] = (int8_t)lo;
                }
            }
            if (l == 0) fx[b] = pow2f(ex - 7);
        }
    }

    struct Lane {
        int g, t, sig, tp;
        bool live;
        uint32_t selA, selB;  // sign-extending byte selects: scale byte sig, 2 + sig
        float lanefac, pw;
    };
    __device__ static Lane lane_setup(int g, int t)
    {
        Lane L;
        L.g = g, L.t = t, L.sig = t >> 1, L.tp = t & 1;
        L.live = (g >> 2) == L.sig;
        const uint32_t a = (uint32_t)L.sig, b = 2u + (uint32_t)L.sig;
        L.selA = a | ((8u | a) << 4) | ((8u | a) << 8) | ((8u | a) << 12);
        L.selB = b | ((8u | b) << 4) | ((8u | b) << 8) | ((8u | b) << 12);
        L.lanefac = L.tp ? 1.0f / 16384.0f : 1.0f;  // pieces 2, 3 weigh 2^-14 of pieces 0, 1
        L.pw = 32.0f * pow2f(-7 * t);               // the offset term of piece t
        return L;
    }

    struct Seg {
        const uint4 *bfl;
        int bq, bb;
        const uint32_t *ofl;
        const float *fxp;
    };
    __device__ static Seg seg_setup(const Lane &L, const uint8_t *prep, const uint8_t *zero, int nb, int)
    {
        Seg s;
        s.bfl = L.live ? reinterpret_cast<const uint4 *>(prep) + 2 * L.g + L.tp : reinterpret_cast<const uint4 *>(zero);
        s.bq = L.live ? 16 : 0, s.bb = L.live ? 64 : 0;
        s.ofl = reinterpret_cast<const uint32_t *>(prep + (size_t)nb * 1024) + (threadIdx.x & 31);
        s.fxp = reinterpret_cast<const float *>(prep + (size_t)nb * 1152);
        return s;
    }

    __device__ static uint32_t code(uint32_t w, uint32_t h, int kk)
    {
        constexpr uint32_t M1 = 0x0F0F0F0Fu, M2 = 0x30303030u;
        switch (kk) {
        case 0: return (w & M1) | ((h << 4) & M2);
        case 1: return (w & M1) | ((h << 2) & M2);
        case 2: return ((w >> 4) & M1) | (h & M2);
        default: return ((w >> 4) & M1) | ((h >> 2) & M2);
        }
    }

    __device__ static void block(const Lane &L, const Seg &S, const uint8_t *slot, int cw, int blk, int nb,
                                 uint64_t *empty, float &acc0, float &acc1)
    {
        const int lane = threadIdx.x & 31;
        const int m = min(SBLK, nb - (blk - cw));  // blocks in this group
        const int QL = 128 * cw + 8 * L.t, QH = 128 * m + 64 * cw + 8 * L.t, SC = 192 * m + 16 * cw,
                  DD = 208 * m + 2 * cw;
        const uint8_t *r0 = slot + L.g * ROWB, *r1 = r0 + 8 * ROWB;
        uint2 qa[2][2], qb[2][2], ha[2], hb[2];
#pragma unroll
        for (int n = 0; n < 2; n++) {
#pragma unroll
            for (int c = 0; c < 2; c++) {
                qa[n][c] = *reinterpret_cast<const uint2 *>(r0 + QL + 64 * n + 32 * c);
                qb[n][c] = *reinterpret_cast<const uint2 *>(r1 + QL + 64 * n + 32 * c);
            }
            ha[n] = *reinterpret_cast<const uint2 *>(r0 + QH + 32 * n);
            hb[n] = *reinterpret_cast<const uint2 *>(r1 + QH + 32 * n);
        }
        const uint4 Sa = *reinterpret_cast<const uint4 *>(r0 + SC), Sb = *reinterpret_cast<const uint4 *>(r1 + SC);
        const unsigned short da = *reinterpret_cast<const unsigned short *>(r0 + DD);
        const unsigned short db = *reinterpret_cast<const unsigned short *>(r1 + DD);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty);
        const uint4 *bp = S.bfl + blk * S.bb;
        const uint4 Bq[4] = {bp[0], bp[S.bq], bp[2 * S.bq], bp[3 * S.bq]};
        const uint32_t ob = S.ofl[blk * 32];
        const uint32_t sa[4] = {Sa.x, Sa.y, Sa.z, Sa.w}, sb[4] = {Sb.x, Sb.y, Sb.z, Sb.w};
        int I0 = 0, I1 = 0, I2 = 0, I3 = 0;
#pragma unroll
        for (int n = 0; n < 2; n++) {
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                const uint2 wa = qa[n][kk & 1], wb = qb[n][kk & 1];
                const int mi = 4 * n + kk;
                const uint4 B = Bq[mi >> 1];
                int D[4] = {0, 0, 0, 0};
                mma_u8s8(D, code(wa.x, ha[n].x, kk), code(wb.x, hb[n].x, kk), code(wa.y, ha[n].y, kk),
                         code(wb.y, hb[n].y, kk), (mi & 1) ? B.z : B.x, (mi & 1) ? B.w : B.y);
                const uint32_t sel = (kk & 1) ? L.selB : L.selA;
                const int sca = (int)prmt_b32(sa[2 * n + (kk >> 1)], 0u, sel);
                const int scb = (int)prmt_b32(sb[2 * n + (kk >> 1)], 0u, sel);
                I0 += sca * D[0];
                I1 += sca * D[1];
                I2 += scb * D[2];
                I3 += scb * D[3];
            }
        }
        // -32 offset: scales (k-slots = sub-blocks 4t..4t+3, as loaded) x sub-block sums of piece t
        int O[4] = {0, 0, 0, 0};
        const uint32_t wa = L.t == 0 ? Sa.x : L.t == 1 ? Sa.y : L.t == 2 ? Sa.z : Sa.w;
        const uint32_t wb = L.t == 0 ? Sb.x : L.t == 1 ? Sb.y : L.t == 2 ? Sb.z : Sb.w;
        mma_s8s8(O, wa, wb, 0u, 0u, ob, 0u);
        const int Ja = 64 * O[0] + O[1], Jb = 64 * O[2] + O[3];
        const float fx = S.fxp[blk];
        const float fa = __half2float(__ushort_as_half(da)) * fx, fb = __half2float(__ushort_as_half(db)) * fx;
        acc0 += fa * (L.lanefac * fmaf(__int2float_rn(I1), 1.0f / 128.0f, __int2float_rn(I0)) -
                      L.pw * __int2float_rn(Ja));
        acc1 += fb * (L.lanefac * fmaf(__int2float_rn(I3), 1.0f / 128.0f, __int2float_rn(I2)) -
                      L.pw * __int2float_rn(Jb));
    }
};

}  // namespace tcmv
}  // namespace sb
