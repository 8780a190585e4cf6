// q4k_mmv.cuh -- Q4_K decode matvec y = W.x on sm_100a: TMA tensor-copy weight
// stream + dequantisation straight into integer tensor-core MMA fragments.
//
// Same block layout and per-sub-block algebra as the reference
// (crates/sosomodel/src/dequant.rs:150-191; gemm.rs:428-461):
//   y[r] = sum_blocks ( d * sum_j sc_j * Sum_l q_l x_l  -  dmin * sum_j m_j * Sum_l x_l )
//
// Numerics.  The 4-bit codes enter a u8 x s8 -> s32 MMA (m16n8k32) as bytes:
// one AND of a qs word gives four low-nibble codes, another four high-nibble
// codes times 16 (not shifted; the 16 is folded into the scales).  x enters as
// four int8 pieces per element, x * 2^(7-ex) = p0 + p1/2^7 + p2/2^14 + p3/2^21
// with 2^ex above the block's max |x| (28 significant bits, every residual
// exact in f32), one piece per B column.  Products and their sums are exact
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
// Work split ("stream-K", deterministic).  Rows are taken 16 at a time (a
// "group", the MMA's M); a stage is (group, 4 consecutive blocks).  The stages
// of the whole matrix, group-major, are split into one contiguous range per
// CTA (row_strip), so every SM gets the same number of bytes whatever the row
// count.  A group cut by a CTA boundary is finished by whichever CTA arrives
// last at its counter, summing the pieces in CTA order; no spinning.
//
// Per CTA: warp 0 is the producer -- one 2-D TMA tensor copy per stage (a
// 16-row x 576-byte box of the weight matrix, seen as u64 elements; rows past
// the end and blocks past a row's end are zero-filled by the TMA unit) into a
// ring of NSLOT slots, issued before griddepcontrol.wait so the stream overlaps
// the previous kernel under programmatic dependent launch.  12 consumer warps
// form 3 teams of 4; team j takes stages j, j+3, ... and within a team warp w
// takes block w of the stage, so three stages are in compute at once.  A warp
// copies its block's bytes to registers and releases the slot before any
// math.  The 576-byte smem row stride is 64 mod 128, so the fragment loads are
// bank-conflict-free.
#pragma once
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace sb {
namespace q4kmmv {

constexpr int SBLK = 4;                   // blocks per stage
constexpr int NCONS = SBLK;               // consumer warps sharing one stage (one block each)
constexpr int NSTREAM = 3;                // stages in flight in compute at once
constexpr int NCW = NCONS * NSTREAM;      // consumer warps
constexpr int THREADS = (NCW + 1) * 32;   // + producer warp
constexpr int NSLOT = 10;                 // ring slots
constexpr int ROWB = SBLK * 144;          // slot row stride: 576 B == 64 mod 128 (conflict-free LDS)
constexpr int SLOTB = 16 * ROWB;          // 9216 B
constexpr int MAX_COLS = 8192;
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
__device__ __forceinline__ bool mbar_wait(uint64_t *b, unsigned parity)
{
    const uint32_t a = smem_u32(b);
    for (unsigned i = 0; i < SPIN_LIMIT; i++) {
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

// 2-D tiled TMA load (no multicast): box at element coords (x = u64 column, y = row).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
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

// Prepared x, per CTA in shared memory, per block b of 256 elements:
//   frag [nb][4 q][16 live lanes][4] u32 -- the int8 x pieces, in the B-fragment
//        order of the u8 x s8 MMAs (see prep_x)
//   mfr  [nb][2 g][4 t] u32 -- f16x2 of the sub-block sums of x, hi (g = 0) and
//        lo (g = 1) halves: the B fragment of the MMA that forms the min terms
//   fx   [nb] f32 -- 2^(ex - 11): weight of piece 0 (and the 1/16 of the high nibbles)
//   fm   [nb] f32 -- 2^(9 + kx): undoes the scaling of the min-term MMA
// (rounded to 16 B: the zero area read as uint4 follows it)
__host__ __device__ inline size_t prep_bytes(int cols) { return ((size_t)(cols / 256) * (1024 + 32 + 8) + 15) & ~(size_t)15; }

// x -> prep.  A warp takes one block (256 elements) at a time; lane l holds
// elements 4l..4l+3 and 128+4l..128+4l+3.  With 2^ex > max|x| over the block,
// each element becomes four int8 pieces, x*2^(7-ex) = p0 + p1/2^7 + p2/2^14 +
// p3/2^21 (28 bits, each residual exact in f32).  Element e of sub-block s,
// piece p, goes to live lane L = 2(4*((s>>1)&1) + p) + (e>>4), register
// 4*(2*(s>>2) + (s&1)) + 2*((e>>3)&1) + ((e>>2)&1), byte e&3.
__device__ __forceinline__ void prep_x(const float *__restrict__ x, int cols, uint8_t *prep, int cw)
{
    const int nb = cols / 256, l = threadIdx.x & 31;
    uint32_t *frag = reinterpret_cast<uint32_t *>(prep);
    unsigned short *mfr = reinterpret_cast<unsigned short *>(prep + (size_t)nb * 1024);
    float *fx = reinterpret_cast<float *>(prep + (size_t)nb * 1056), *fm = fx + nb;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    for (int b = cw; b < nb; b += NCW) {
        const float4 va = x4[b * 64 + l], vb = x4[b * 64 + 32 + l];
        float mx = fmaxf(fmaxf(fmaxf(fabsf(va.x), fabsf(va.y)), fmaxf(fabsf(va.z), fabsf(va.w))),
                         fmaxf(fmaxf(fabsf(vb.x), fabsf(vb.y)), fmaxf(fabsf(vb.z), fabsf(vb.w))));
        float sa = (va.x + va.y) + (va.z + va.w), sbv = (vb.x + vb.y) + (vb.z + vb.w);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            sa += __shfl_xor_sync(0xffffffffu, sa, o);
            sbv += __shfl_xor_sync(0xffffffffu, sbv, o);
        }
        // 2^ex > max|x| (ex from the biased exponent of the max), clamped for zero / non-finite input
        const uint32_t mxb = __float_as_uint(mx);
        int ex = (int)(mxb >> 23) - 126;
        ex = (mxb == 0u || mxb >= 0x7f800000u) ? 0 : ex < -100 ? -100 : ex > 100 ? 100 : ex;
        const float scl = __uint_as_float((uint32_t)(127 + 7 - ex) << 23);
        auto pieces = [&](float4 v4, int n) {
            const int sblk = n >> 5, e = n & 31;
            const int sig = (sblk >> 1) & 1, q = 2 * (sblk >> 2) + (sblk & 1);
            const int word = 2 * ((e >> 3) & 1) + ((e >> 2) & 1), tp = e >> 4;
            const float xs[4] = {v4.x, v4.y, v4.z, v4.w};
            uint32_t pk[4] = {0u, 0u, 0u, 0u};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                float v = xs[i] * scl;
#pragma unroll
                for (int pc = 0; pc < 4; pc++) {
                    float r = rintf(v);
                    r = fminf(fmaxf(r, -127.0f), 127.0f);
                    pk[pc] |= ((uint32_t)__float2int_rn(r) & 0xFFu) << (8 * i);
                    v = (v - r) * 128.0f;
                }
            }
#pragma unroll
            for (int pc = 0; pc < 4; pc++) {
                const int L = 2 * (4 * sig + pc) + tp;
                frag[((b * 4 + q) * 16 + L) * 4 + word] = pk[pc];
            }
        };
        pieces(va, 4 * l);
        pieces(vb, 128 + 4 * l);
        // sub-block sums -> f16 hi/lo with one power-of-two scale per block (max below 2^15)
        float smx = fmaxf(fabsf(sa), fabsf(sbv));
#pragma unroll
        for (int o = 8; o < 32; o <<= 1) smx = fmaxf(smx, __shfl_xor_sync(0xffffffffu, smx, o));
        const uint32_t smb = __float_as_uint(smx);
        int kx = (int)(smb >> 23) - 126;
        kx = (smb == 0u || smb >= 0x7f800000u) ? 0 : kx < -100 ? -100 : kx > 100 ? 100 : kx;
        const float ms = __uint_as_float((uint32_t)(127 + 15 - kx) << 23);
        if ((l & 7) == 0) {
            const float sv[2] = {sa, sbv};
#pragma unroll
            for (int c = 0; c < 2; c++) {
                const int sidx = 4 * c + (l >> 3);
                const float v = sv[c] * ms;
                const __half hi = __float2half_rn(v), lo = __float2half_rn(v - __half2float(hi));
                mfr[((b * 2 + 0) * 4 + (sidx >> 1)) * 2 + (sidx & 1)] = __half_as_ushort(hi);
                mfr[((b * 2 + 1) * 4 + (sidx >> 1)) * 2 + (sidx & 1)] = __half_as_ushort(lo);
            }
        }
        if (l == 0) {
            fx[b] = __uint_as_float((uint32_t)(127 + ex - 11) << 23);
            fm[b] = __uint_as_float((uint32_t)(127 + 9 + kx) << 23);
        }
    }
}

struct Smem {
    // ring + prepared x + per-group partials + barriers, carved from dynamic smem
    uint8_t *ring;    // NSLOT * SLOTB
    uint8_t *prep;    // prep_bytes(cols): frag, fb, sx
    uint8_t *zero;    // 64 B of zeros
    float *part;      // [ngroups_cta][NCW][16]
    uint64_t *full;   // [NSLOT]
    uint64_t *empty;  // [NSLOT]
};

__host__ __device__ inline size_t smem_bytes(int cols, int max_groups)
{
    return (size_t)NSLOT * SLOTB + prep_bytes(cols) + 64 + (size_t)max_groups * NCW * 64 + 2 * NSLOT * 8 + 64;
}

__device__ __forceinline__ Smem carve(uint8_t *base, int cols, int max_groups)
{
    Smem s;
    size_t o = 0;
    s.ring = base;
    o += (size_t)NSLOT * SLOTB;
    s.prep = base + o;
    o += prep_bytes(cols);
    s.zero = base + o;  // 64 zero bytes: the B fragment of lanes that carry no x
    o += 64;
    s.part = reinterpret_cast<float *>(base + o);
    o += (size_t)max_groups * NCW * 64;
    o = (o + 7) & ~(size_t)7;
    s.full = reinterpret_cast<uint64_t *>(base + o);
    s.empty = s.full + NSLOT;
    return s;
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ int owner_of(int unit, int total, int n)
{
    // inverse of row_strip: which of n parts holds `unit`
    const int base = total / n, rem = total - base * n;
    const int big = rem * (base + 1);
    return unit < big ? unit / (base + 1) : rem + (base ? (unit - big) / base : 0);
}

// One launch serves a batch of independent matvecs (the reference's
// matvec_lote: several matvecs, one wait).  Their stages are numbered one
// after another; the CTAs split that global range, so the batch streams as one.
constexpr int MAXB = 40;

struct __align__(64) MatDesc {
    CUtensorMap map;        // weights as [rows][row_bytes/8] u64, box 16 x 72
    const float *x;
    float *y;
    int rows, cols, spg;    // spg: stages per 16-row group
    int st_begin, cnt_off;  // first global stage; first counter of its groups
};

struct Batch {
    MatDesc d[MAXB];
    int n, total;            // matrices, stages
    int max_cols, max_groups;  // shared-memory capacities (prep, partial table)
};

__global__ void __launch_bounds__(THREADS, 1) q4k_mmv_kernel(const __grid_constant__ Batch B, Ws ws)
{
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Smem s = carve(smem_raw, B.max_cols, B.max_groups);
    int st0, st1;
    row_strip(B.total, blockIdx.x, gridDim.x, st0, st1);
    const int nst = st1 - st0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // matrices touched: m_first .. m_last
    int m_first = 0;
    while (m_first + 1 < B.n && B.d[m_first + 1].st_begin <= st0) m_first++;
    int m_last = m_first;
    while (nst > 0 && m_last + 1 < B.n && B.d[m_last + 1].st_begin < st1) m_last++;

    if (threadIdx.x == 0) {
        for (int k = 0; k < NSLOT; k++) {
            mbar_init(&s.full[k], 1);
            mbar_init(&s.empty[k], NCONS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < 16) reinterpret_cast<float *>(s.zero)[threadIdx.x] = 0.0f;
    __syncthreads();
    // Dependents may launch now: they only read what this grid writes after their
    // own griddepcontrol.wait, which waits for this grid to complete.
    griddep_launch();

    bool failed = false;
    if (warp == 0) {
        // ---------------- producer: weights do not depend on the previous kernel, so the
        // whole stream runs without griddepcontrol.wait
        if (lane == 0 && nst > 0) {
            int mi = m_first, slot = 0;
            unsigned phase = 0;  // parity of the empty-barrier phase to wait for
            const MatDesc *d = &B.d[mi];
            int ls = st0 - d->st_begin, G = ls / d->spg, j = ls - G * d->spg;
            int mend = d->st_begin + d->spg * ((d->rows + 15) >> 4);
            asm volatile("prefetch.tensormap [%0];" ::"l"(&d->map) : "memory");
            for (int k = 0; k < nst; k++) {
                if (st0 + k == mend) {  // next matrix of the batch
                    d = &B.d[++mi];
                    G = 0, j = 0;
                    mend = d->st_begin + d->spg * ((d->rows + 15) >> 4);
                    asm volatile("prefetch.tensormap [%0];" ::"l"(&d->map) : "memory");
                }
                if (k >= NSLOT && !mbar_wait(&s.empty[slot], phase)) {
                    failed = true;
                    break;
                }
                mbar_expect_tx_arrive(&s.full[slot], (unsigned)SLOTB);  // full box, zero-filled past the ends
                tma_load_2d(s.ring + slot * SLOTB, &d->map, j * SBLK * 18, G * 16, &s.full[slot]);
                if (++j == d->spg) j = 0, G++;
                if (++slot == NSLOT) {
                    slot = 0;
                    if (k >= NSLOT) phase ^= 1u;  // stages 2*NSLOT.. wait for the second use of a slot, ...
                }
            }
            if (failed) set_dev_error(0x51u);
        }
        __syncwarp();
    } else {
        // ---------------- consumers
        const int cwg = warp - 1;  // 0 .. NCW-1
        const int team = cwg / NCONS, cw = cwg % NCONS, g = lane >> 2, t = lane & 3, q2 = t >> 1;
        // B columns are (sub-block slot g/4, piece g%4): a lane carries x only where its
        // k-slots (sub-block slot t/2) meet its column
        const bool live = (g >> 2) == q2, mlive = g < 2;
        const uint8_t *ring_lane = s.ring + g * ROWB + cw * 144;  // + slot * SLOTB
        const int qoff = 16 + t * 16;                               // + 64 * duo
        const int sc_sh = 16 * q2;
        // min-term A fragment: m of sub-blocks 2t, 2t+1 as f16 subnormals (byte -> u16 lane)
        const uint32_t sel_m = (uint32_t)((2 * t) & 3) | 0x40u | ((uint32_t)(((2 * t) & 3) + 1) << 8) | 0x4000u;
        const float lanefac = (t & 1) ? 1.0f / 16384.0f : 1.0f;  // pieces 2, 3 weigh 2^-14 of pieces 0, 1
        griddep_wait();  // x of every matrix is written by the previous kernel
        for (int mi = m_first; mi <= m_last && nst > 0; mi++) {
            const MatDesc &d = B.d[mi];
            const int cols = d.cols, nb = cols / 256, spg = d.spg;
            const int mtot = spg * ((d.rows + 15) >> 4);
            const int ka = max(st0, d.st_begin) - st0, kb = min(st1, d.st_begin + mtot) - st0;  // CTA-local stages
            const int gs0 = (ka + st0 - d.st_begin) / spg, gs1 = (kb - 1 + st0 - d.st_begin) / spg;
            const int ng = gs1 - gs0 + 1;
            // x -> prep (frag, scales, sums) and a clean partial table for this segment
            prep_x(d.x, cols, s.prep, cwg);
            for (int i = cwg * 32 + lane; i < ng * NCW * 16; i += NCW * 32) s.part[i] = 0.0f;
            asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
            // x-side fragments of this lane (lanes without x read zeros: stride 0 into s.zero)
            const uint4 *bfl = live ? reinterpret_cast<const uint4 *>(s.prep) + 2 * g + (t & 1)
                                    : reinterpret_cast<const uint4 *>(s.zero);
            const int bq = live ? 16 : 0, bb = live ? 64 : 0;
            const uint32_t *mfl = mlive ? reinterpret_cast<const uint32_t *>(s.prep + (size_t)nb * 1024) + g * 4 + t
                                        : reinterpret_cast<const uint32_t *>(s.zero);
            const int mb = mlive ? 8 : 0;
            const float *fxp = reinterpret_cast<const float *>(s.prep + (size_t)nb * 1056), *fmp = fxp + nb;
            float acc0 = 0.0f, acc1 = 0.0f;
            int cur = -1;
            const int k0 = ka + team;
            int slot = k0 % NSLOT, G = (k0 + st0 - d.st_begin) / spg, j = (k0 + st0 - d.st_begin) - G * spg;
            unsigned parity = (k0 / NSLOT) & 1;
            for (int k = k0; k < kb && !failed; k += NSTREAM) {
                if (k != k0) {  // advance by NSTREAM stages
                    slot += NSTREAM;
                    if (slot >= NSLOT) slot -= NSLOT, parity ^= 1u;
                    j += NSTREAM;
                    while (j >= spg) j -= spg, G++;
                }
                if (!mbar_wait(&s.full[slot], parity)) {
                    failed = true;
                    set_dev_error(0x52u);
                    break;
                }
                const int blk = j * SBLK + cw;
                bool released = false;
                if (G != cur) {
                    if (cur >= 0) {
                        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
                        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
                        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
                        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
                        if (t == 0) {
                            float *p = s.part + ((cur - gs0) * NCW + cwg) * 16;
                            p[g] = acc0;
                            p[g + 8] = acc1;
                        }
                    }
                    cur = G;
                    acc0 = acc1 = 0.0f;
                }
                if (blk < nb) {
                    const uint8_t *r0p = ring_lane + slot * SLOTB, *r1p = r0p + 8 * ROWB;
                    const uint4 h0 = *reinterpret_cast<const uint4 *>(r0p);
                    const uint4 h1 = *reinterpret_cast<const uint4 *>(r1p);
                    // rows g / g+8: 16 bytes of pair 2*duo + t/2 each (bytes 16*(t&1).. of the pair)
                    const uint4 qa0 = *reinterpret_cast<const uint4 *>(r0p + qoff);
                    const uint4 qa1 = *reinterpret_cast<const uint4 *>(r0p + qoff + 64);
                    const uint4 qb0 = *reinterpret_cast<const uint4 *>(r1p + qoff);
                    const uint4 qb1 = *reinterpret_cast<const uint4 *>(r1p + qoff + 64);
                    // The stage's bytes are in registers: hand the slot back to the producer
                    // now (arrive has release semantics, so these reads precede its refill).
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s.empty[slot]);
                    released = true;
                    const uint4 *bp = bfl + blk * bb;
                    const uint4 B0 = bp[0], B1 = bp[bq], B2 = bp[2 * bq], B3 = bp[3 * bq];
                    const uint32_t mbv = mfl[blk * mb];
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
                        const uint32_t s0 = S0 >> sc_sh, s1 = S1 >> sc_sh;
                        // low-nibble sub-blocks carry codes x1, high-nibble ones x16: scale the former by 16
                        c[0] = (int)((s0 << 4) & 0xFF0u);
                        c[1] = (int)((s0 >> 8) & 0xFFu);
                        c[2] = (int)((s1 << 4) & 0xFF0u);
                        c[3] = (int)((s1 >> 8) & 0xFFu);
                        am = __byte_perm(t < 2 ? M0 : M1, 0u, sel_m);
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
                    const float fxl = fxp[blk] * lanefac, fml = fmp[blk];
                    acc0 += (dn0.x * fxl) * fmaf(__int2float_rn(I01), 1.0f / 128.0f, __int2float_rn(I00)) -
                            (dn0.y * fml) * (dm[0] + dm[1]);
                    acc1 += (dn1.x * fxl) * fmaf(__int2float_rn(I11), 1.0f / 128.0f, __int2float_rn(I10)) -
                            (dn1.y * fml) * (dm[2] + dm[3]);
                }
                if (!released) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s.empty[slot]);
                }
            }
            if (cur >= 0) {
                acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
                acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
                acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
                acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
                if (t == 0) {
                    float *p = s.part + ((cur - gs0) * NCW + cwg) * 16;
                    p[g] = acc0;
                    p[g + 8] = acc1;
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
            // segment epilogue: sum the consumer warps' pieces per group (fixed order)
            const bool head_cut = mi == m_first && (st0 - d.st_begin) % spg != 0;
            const bool tail_cut = mi == m_last && (st1 - d.st_begin) % spg != 0 && st1 < d.st_begin + mtot;
            for (int i = cwg * 32 + lane; i < ng * 16; i += NCW * 32) {
                const int gl = i >> 4, r = i & 15, row = (gs0 + gl) * 16 + r;
                float v = 0.0f;
                for (int w = 0; w < NCW; w++) v += s.part[(gl * NCW + w) * 16 + r];
                const bool cut = (gl == 0 && head_cut) || (gl == ng - 1 && tail_cut);
                if (!cut) {
                    if (row < d.rows) d.y[row] = v;
                } else {
                    // side 0: the group holding this CTA's first stage, side 1: any other (its last)
                    const int ga = d.st_begin + (gs0 + gl) * spg;
                    ws.part[(blockIdx.x * 2 + ((st0 >= ga && st0 < ga + spg) ? 0 : 1)) * 16 + r] = v;
                    __threadfence();
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
        }
    }
    if (failed) {
        // let every TMA copy issued into this CTA's shared memory land before exiting (bounded)
        if (warp == 0 && lane == 0)
            for (int k = nst > NSLOT ? nst - NSLOT : 0; k < nst; k++) mbar_wait(&s.full[k % NSLOT], (k / NSLOT) & 1);
    }
    __syncthreads();
    if (nst <= 0) return;

    // ---------------- groups cut by CTA boundaries: the last CTA to arrive at a group's
    // counter sums the pieces in CTA order.  Both sides in one round trip.
    __shared__ int last_flag[2];
    __shared__ int side_g[2], side_ca[2], side_cb[2], side_m[2];
    if (threadIdx.x < 2) {
        const int side = threadIdx.x;
        const int mi = side == 0 ? m_first : m_last;
        const MatDesc &d = B.d[mi];
        const int mtot = d.spg * ((d.rows + 15) >> 4);
        const int ls0 = st0 - d.st_begin, ls1 = st1 - d.st_begin;  // stage range relative to the matrix
        const bool head_cut = ls0 % d.spg != 0;
        const bool tail_cut = ls1 % d.spg != 0 && ls1 < mtot;
        // one group cut on both sides of a one-group range is side 0's job
        const bool single = m_first == m_last && (ls0 / d.spg) == ((ls1 - 1) / d.spg);
        const bool mine = side == 0 ? head_cut || (single && tail_cut) : (tail_cut && !single);
        int flag = 0;
        if (mine) {
            const int G = side == 0 ? ls0 / d.spg : (ls1 - 1) / d.spg;
            const int ga = d.st_begin + G * d.spg;
            const int c_a = owner_of(ga, B.total, gridDim.x), c_b = owner_of(ga + d.spg - 1, B.total, gridDim.x);
            flag = atomicAdd(&ws.cnt[d.cnt_off + G], 1u) == (unsigned)(c_b - c_a);
            side_g[side] = G, side_ca[side] = c_a, side_cb[side] = c_b, side_m[side] = mi;
        }
        last_flag[side] = flag;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int side = threadIdx.x >> 4, r = threadIdx.x & 15;
        if (last_flag[side]) {
            __threadfence();
            const MatDesc &d = B.d[side_m[side]];
            const int G = side_g[side], ga = d.st_begin + G * d.spg, ge = ga + d.spg;
            float v = 0.0f;
            for (int c = side_ca[side]; c <= side_cb[side]; c++) {
                int cs0, cs1;
                row_strip(B.total, c, gridDim.x, cs0, cs1);
                // CTA c stored G as side 0 if its range starts inside G, else as side 1
                v += __ldcg(&ws.part[(c * 2 + ((cs0 >= ga && cs0 < ge) ? 0 : 1)) * 16 + r]);
            }
            if (G * 16 + r < d.rows) d.y[G * 16 + r] = v;
            if (r == 0) ws.cnt[d.cnt_off + G] = 0u;
        }
    }
}

// Workspace layout (fixed offsets, whatever the shape, because one workspace
// serves every launch on a stream): [cnt: CNT_MAX u32, zero between launches]
// [part: grid*2*16 f32].  Zeroed once when allocated.
constexpr int CNT_MAX = 1 << 16;  // groups of 16 rows: up to 1M rows
inline size_t ws_part_off() { return (size_t)CNT_MAX * 4; }
inline size_t ws_bytes(int grid) { return ws_part_off() + (size_t)grid * 2 * 16 * 4 + 256; }

// Launch on `stream`; ws must hold ws_bytes(rows, grid) bytes, zeroed before first use
// (the kernel leaves its counters at zero).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn()
{
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

// Weights as a [rows][row_bytes/8] u64 tensor, box = 16 rows x 72 u64 (4 blocks).
inline int make_map(CUtensorMap *m, const void *w, int rows, int cols)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return -6;
    const cuuint64_t rb = (cuuint64_t)(cols / 256) * 144;
    cuuint64_t dims[2] = {rb / 8, (cuuint64_t)rows};
    cuuint64_t strides[1] = {rb};
    cuuint32_t box[2] = {SBLK * 18, 16};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(w), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -7;
}

// Tensor maps are pure functions of (pointer, shape); keep the last few.
inline int cached_map(CUtensorMap *out, const void *w, int rows, int cols)
{
    struct E {
        const void *w;
        int rows, cols;
        CUtensorMap m;
    };
    static E cache[64];
    static int next = 0;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    for (auto &e : cache)
        if (e.w == w && e.rows == rows && e.cols == cols) {
            *out = e.m;
            return 0;
        }
    E &e = cache[next];
    next = (next + 1) % 64;
    const int rc = make_map(&e.m, w, rows, cols);
    if (rc) {
        e.w = nullptr;
        return rc;
    }
    e.w = w;
    e.rows = rows;
    e.cols = cols;
    *out = e.m;
    return 0;
}

struct MatOp {
    const void *w;
    int rows, cols;
    const float *x;
    float *y;
};

// Shared memory for a batch over `grid` CTAs (0 if it exceeds the SM).
inline size_t batch_smem(const MatOp *ops, int n, int grid, int *max_cols, int *max_groups)
{
    long long total = 0;
    int mc = 0;
    for (int i = 0; i < n; i++) {
        const int spg = (ops[i].cols / 256 + SBLK - 1) / SBLK;
        total += (long long)spg * ((ops[i].rows + 15) / 16);
        mc = ops[i].cols > mc ? ops[i].cols : mc;
    }
    const long long per = (total + grid - 1) / grid;
    int mg = 1;
    for (int i = 0; i < n; i++) {
        const int spg = (ops[i].cols / 256 + SBLK - 1) / SBLK, groups = (ops[i].rows + 15) / 16;
        const long long g = per / spg + 2;
        const int gi = (int)(g < groups ? g : groups);
        mg = gi > mg ? gi : mg;
    }
    *max_cols = mc;
    *max_groups = mg;
    return (size_t)NSLOT * SLOTB + prep_bytes(mc) + 64 + (size_t)mg * NCW * 64 + 2 * NSLOT * 8 + 64;
}

// Launch a batch of up to MAXB independent Q4_K matvecs on `stream`; ws holds
// ws_bytes() bytes, zeroed before its first use (the kernel leaves it zeroed).
inline int launch_batch(const MatOp *ops, int n, void *ws, int grid, int pdl, cudaStream_t stream)
{
    if (n < 1 || n > MAXB) return -1;
    static Batch b;  // large: built host-side, passed by value as the kernel parameter
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    int st = 0, cnt = 0;
    for (int i = 0; i < n; i++) {
        const MatOp &o = ops[i];
        if (o.cols > MAX_COLS || o.cols % 256 || o.rows < 1) return -1;
        MatDesc &d = b.d[i];
        const int mrc = cached_map(&d.map, o.w, o.rows, o.cols);
        if (mrc) return mrc;
        d.x = o.x;
        d.y = o.y;
        d.rows = o.rows;
        d.cols = o.cols;
        d.spg = (o.cols / 256 + SBLK - 1) / SBLK;
        d.st_begin = st;
        d.cnt_off = cnt;
        st += d.spg * ((o.rows + 15) / 16);
        cnt += (o.rows + 15) / 16;
    }
    if (cnt > CNT_MAX) return -1;
    b.n = n;
    b.total = st;
    const size_t smem = batch_smem(ops, n, grid, &b.max_cols, &b.max_groups);
    if (smem > 227 * 1024) return -5;
    static size_t smem_set[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return -3;
    if (smem > smem_set[dev]) {
        if (cudaFuncSetAttribute(q4k_mmv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return -3;
        smem_set[dev] = smem;
    }
    uint8_t *wsb = reinterpret_cast<uint8_t *>(ws);
    Ws wsd;
    wsd.cnt = reinterpret_cast<unsigned *>(wsb);
    wsd.part = reinterpret_cast<float *>(wsb + ws_part_off());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, q4k_mmv_kernel, b, wsd) == cudaSuccess ? 0 : -4;
}

// As launch_batch, with the scratch given as explicit counter / partial pointers
// (used by the entry point that allocates nothing, whose scratch is a fixed array).
inline int launch_batch_with(const MatOp *ops, int n, Ws wsd, int grid, int pdl, cudaStream_t stream)
{
    if (n < 1 || n > MAXB) return -1;
    static Batch b;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    int st = 0, cnt = 0;
    for (int i = 0; i < n; i++) {
        const MatOp &o = ops[i];
        if (o.cols > MAX_COLS || o.cols % 256 || o.rows < 1) return -1;
        MatDesc &d = b.d[i];
        const int mrc = cached_map(&d.map, o.w, o.rows, o.cols);
        if (mrc) return mrc;
        d.x = o.x;
        d.y = o.y;
        d.rows = o.rows;
        d.cols = o.cols;
        d.spg = (o.cols / 256 + SBLK - 1) / SBLK;
        d.st_begin = st;
        d.cnt_off = cnt;
        st += d.spg * ((o.rows + 15) / 16);
        cnt += (o.rows + 15) / 16;
    }
    b.n = n;
    b.total = st;
    const size_t smem = batch_smem(ops, n, grid, &b.max_cols, &b.max_groups);
    if (smem > 227 * 1024) return -5;
    // Read the kernel's current dynamic shared-memory limit on every call and only
    // ever RAISE it: launch_batch keeps its own record of what it set, so this
    // launcher neither lowers the limit under it nor trusts a record of its own.
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, q4k_mmv_kernel) != cudaSuccess) return -3;
    if ((size_t)fa.maxDynamicSharedSizeBytes < smem &&
        cudaFuncSetAttribute(q4k_mmv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return -3;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, q4k_mmv_kernel, b, wsd) == cudaSuccess ? 0 : -4;
}

inline bool fits(const MatOp *ops, int n, int grid)
{
    int mc, mg;
    for (int i = 0; i < n; i++)
        if (ops[i].cols > MAX_COLS || ops[i].cols % 256) return false;
    return batch_smem(ops, n, grid, &mc, &mg) <= 227 * 1024;
}

}  // namespace q4kmmv
}  // namespace sb
