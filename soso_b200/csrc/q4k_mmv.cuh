// q4k_mmv.cuh -- Q4_K decode matvec y = W.x on sm_100a: TMA bulk-copy weight
// stream + dequantisation straight into mma.sync bf16 fragments.
//
// Same block layout and per-sub-block algebra as the reference
// (crates/sosomodel/src/dequant.rs:150-191; gemm.rs:428-461):
//   y[r] = sum_blocks sum_j ( d*sc_j * Sum_l q_l x_l  -  dmin*m_j * Sum_l x_l )
// Only the inner Sum_l q_l x_l is done by the tensor core; scales, mins and
// the row accumulation are f32 on the CUDA cores.
//
// Numerics.  A code q (0..15) enters the MMA as the f16 bit pattern q itself,
// i.e. the subnormal q * 2^-24 -- exact, no offset to cancel.  x enters as two
// f16 columns, hi = f16(x * 2^s) and lo = f16(x * 2^s - hi) (22 significant
// bits), with a power-of-two scale 2^s chosen per 32-element sub-block so the
// largest element sits just below 2^15.  Products are exact and accumulate in
// f32 inside the MMA; the epilogue multiplies by 2^(24 - s).  Each CTA builds
// these x-side operands (fragments, scales, sub-block sums of x) in shared
// memory while its weight stream is already in flight.
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
// takes block w of the stage, so three stages are in compute at once.  Within
// a block the two half-blocks and the even/odd MMAs form four independent
// accumulation chains, so the tensor-core latency overlaps.  A
// lane (g = lane/4, t = lane%4) holds rows g and g+8, chunk t: 8 m16n8k16 MMAs
// give, in D column pair (2t, 2t+1), the hi/lo partial sums of sub-block t of
// that half-block for both rows.  The 576-byte smem row stride is 64 mod 128,
// so the fragment loads are bank-conflict-free.
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

// Lanes of an MMA whose B column meets their own k-slots: lane (g, t) with
// g/4 == t/2.  Only they carry x; the other 16 lanes pass zeros.  Compact id:
__host__ __device__ __forceinline__ int frag_lane(int g, int t) { return (g >> 2) * 8 + (g & 3) * 2 + (t & 1); }
__host__ __device__ __forceinline__ bool frag_live(int g, int t) { return (g >> 2) == (t >> 1); }

// Code registers, as f16 subnormals without shifting where possible: for a
// qs word w (bytes b0..b3), MMA m = 2*iw + sub uses bytes (sub, sub+2):
//   low nibbles  (w >> 8*sub) & 0x000F000F  -> q * 2^-24
//   high nibbles (w >> 8*sub) & 0x00F000F0  -> q * 2^-20 (the factor 16 is
//   folded into the scale of the odd, high-nibble sub-blocks)

// Prepared x, per CTA in shared memory:
//   frag [HB][16 live lanes][8 MMAs][2] u32 -- (b0, b1) f16x2 of that lane; the
//        one its column does not use is 0
//   fb   [HB*4] f32 -- 2^(24 - s) per sub-block (2^(20 - s) for odd sub-blocks)
//   sx   [HB*4] f32 -- sum of x per sub-block (for the -dmin*m term)
__host__ __device__ inline size_t prep_bytes(int cols) { return (size_t)(cols / 128) * 1024 + (size_t)cols / 32 * 8; }

// x -> prep.  A warp takes one half-block (128 elements, 4 sub-blocks) at a
// time; lane l loads elements 4l..4l+3, so sub-block s = l/8 and element
// e = 4(l%8) + i of it.  Sub-block s is the low (s even) or high (s odd)
// nibbles of pair s/2, element e is byte e of the pair: chunk t = 2(s/2) + e/16,
// word (e%16)/4 = l%4, byte e%4 = i: MMA m = 2(l%4) + i%2, half i/2 of the
// f16x2; its hi piece goes to column g = 2s, lo piece to g = 2s+1, register
// b0 (s even) or b1 (s odd).  Per-sub-block max and sum over 8 lanes.
__device__ __forceinline__ void prep_x(const float *__restrict__ x, int cols, uint8_t *prep, int cw)
{
    const int HB = cols / 128, l = threadIdx.x & 31, s = l >> 3, q = l & 7;
    const int t = 2 * (s >> 1) + (q >> 2), m0 = 2 * (l & 3);
    // u16 offsets within one half-block (512 u16) for element i = 0; i adds (i%2)*4 + i/2
    const int o_hi = ((frag_lane(2 * s, t) * 8 + m0) * 2 + (s & 1)) * 2;
    const int o_lo = ((frag_lane(2 * s + 1, t) * 8 + m0) * 2 + (s & 1)) * 2;
    unsigned short *f16p = reinterpret_cast<unsigned short *>(prep);
    float *fb = reinterpret_cast<float *>(prep + (size_t)HB * 1024);
    // zero the frag area (half of it is never written: the b-register a column does not use)
    uint4 *z = reinterpret_cast<uint4 *>(prep);
    for (int i = cw * 32 + l; i < HB * 64; i += NCW * 32) z[i] = make_uint4(0, 0, 0, 0);
    float4 v[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int hb = cw + r * NCW;
        v[r] = hb < HB ? *reinterpret_cast<const float4 *>(x + hb * 128 + 4 * l) : make_float4(0, 0, 0, 0);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
    auto one = [&](float4 a, int hb) {
        float mx = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w)));
        float sm = (a.x + a.y) + (a.z + a.w);
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            sm += __shfl_xor_sync(0xffffffffu, sm, o);
        }
        const uint32_t mxb = __float_as_uint(mx);
        // 2^(E-126) > max|x| for a normal max with biased exponent E; scale it below 2^15
        int ex = (int)(mxb >> 23) - 126;
        ex = (mxb == 0u || mxb >= 0x7f800000u) ? 0 : ex < -100 ? -100 : ex > 100 ? 100 : ex;
        const float scale = __uint_as_float((uint32_t)(127 + 15 - ex) << 23);
        const int c = hb * 4 + s;
        if (q == 0) {
            fb[c] = __uint_as_float((uint32_t)(127 + 9 + ex - (s & 1) * 4) << 23);  // 2^(24 - (15 - ex)) / 16^(s&1)
            fb[HB * 4 + c] = sm;
        }
        unsigned short *hp = f16p + (size_t)hb * 512;
        const float xa[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float xv = xa[i] * scale;
            const __half hi = __float2half_rn(xv), lo = __float2half_rn(xv - __half2float(hi));
            const int d = (i & 1) * 4 + (i >> 1);
            hp[o_hi + d] = __half_as_ushort(hi);
            hp[o_lo + d] = __half_as_ushort(lo);
        }
    };
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int hb = cw + r * NCW;
        if (hb < HB) one(v[r], hb);
    }
    for (int hb = cw + 4 * NCW; hb < HB; hb += NCW) one(*reinterpret_cast<const float4 *>(x + hb * 128 + 4 * l), hb);
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
        const int team = cwg / NCONS, cw = cwg % NCONS, g = lane >> 2, t = lane & 3, sh = 8 * t;
        const bool live = frag_live(g, t);
        const int fstride = live ? 1024 : 0;
        const uint8_t *ring_lane = s.ring + g * ROWB + cw * 144;  // + slot * SLOTB
        const int qoff = 16 + t * 16;
        griddep_wait();  // x of every matrix is written by the previous kernel
        for (int mi = m_first; mi <= m_last && nst > 0; mi++) {
            const MatDesc &d = B.d[mi];
            const int cols = d.cols, nb = cols / 256, spg = d.spg, HB = cols / 128;
            const int mtot = spg * ((d.rows + 15) >> 4);
            const int ka = max(st0, d.st_begin) - st0, kb = min(st1, d.st_begin + mtot) - st0;  // CTA-local stages
            const int gs0 = (ka + st0 - d.st_begin) / spg, gs1 = (kb - 1 + st0 - d.st_begin) / spg;
            const int ng = gs1 - gs0 + 1;
            // x -> prep (frag, scales, sums) and a clean partial table for this segment
            prep_x(d.x, cols, s.prep, cwg);
            for (int i = cwg * 32 + lane; i < ng * NCW * 16; i += NCW * 32) s.part[i] = 0.0f;
            asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
            const uint8_t *fragl = live ? s.prep + frag_lane(g, t) * 64 : s.zero;
            const float *fbt = reinterpret_cast<const float *>(s.prep + (size_t)HB * 1024) + t, *sxt = fbt + HB * 4;
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
                    uint4 qa[2], qb[2], Bv[2][4];
#pragma unroll
                    for (int half = 0; half < 2; half++) {
                        qa[half] = *reinterpret_cast<const uint4 *>(r0p + qoff + half * 64);
                        qb[half] = *reinterpret_cast<const uint4 *>(r1p + qoff + half * 64);
                    }
                    // The stage's bytes are in registers: hand the slot back to the producer
                    // now (arrive has release semantics, so these reads precede its refill).
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s.empty[slot]);
                    released = true;
                    const float2 dn0 = __half22float2(*reinterpret_cast<const __half2 *>(&h0.x));
                    const float2 dn1 = __half22float2(*reinterpret_cast<const __half2 *>(&h1.x));
                    const uint32_t x0 = h0.y >> sh, y0 = h0.z >> sh, z0 = h0.w >> sh;
                    const uint32_t x1 = h1.y >> sh, y1 = h1.z >> sh, z1 = h1.w >> sh;
                    const uint8_t *fr = fragl + blk * 2 * fstride;
                    const float *fbb = fbt + blk * 8, *sxb = sxt + blk * 8;
#pragma unroll
                    for (int half = 0; half < 2; half++) {
                        const uint4 *fp = reinterpret_cast<const uint4 *>(fr + half * fstride);
#pragma unroll
                        for (int q = 0; q < 4; q++) Bv[half][q] = fp[q];
                    }
                    // four independent chains: (half, byte pair 0/2 vs 1/3)
                    float dacc[2][2][4];
#pragma unroll
                    for (int h = 0; h < 2; h++)
#pragma unroll
                        for (int p = 0; p < 2; p++)
#pragma unroll
                            for (int i = 0; i < 4; i++) dacc[h][p][i] = 0.0f;
#pragma unroll
                    for (int iw = 0; iw < 4; iw++) {
#pragma unroll
                        for (int half = 0; half < 2; half++) {
                            const uint32_t wa[4] = {qa[half].x, qa[half].y, qa[half].z, qa[half].w};
                            const uint32_t wb[4] = {qb[half].x, qb[half].y, qb[half].z, qb[half].w};
                            const uint32_t bb[16] = {Bv[half][0].x, Bv[half][0].y, Bv[half][0].z, Bv[half][0].w,
                                                     Bv[half][1].x, Bv[half][1].y, Bv[half][1].z, Bv[half][1].w,
                                                     Bv[half][2].x, Bv[half][2].y, Bv[half][2].z, Bv[half][2].w,
                                                     Bv[half][3].x, Bv[half][3].y, Bv[half][3].z, Bv[half][3].w};
                            const uint32_t a = wa[iw], b = wb[iw], a8 = a >> 8, b8 = b >> 8;
                            mma_f16(dacc[half][0], a & 0x000F000Fu, b & 0x000F000Fu, a & 0x00F000F0u,
                                    b & 0x00F000F0u, bb[(2 * iw) * 2], bb[(2 * iw) * 2 + 1]);
                            mma_f16(dacc[half][1], a8 & 0x000F000Fu, b8 & 0x000F000Fu, a8 & 0x00F000F0u,
                                    b8 & 0x00F000F0u, bb[(2 * iw + 1) * 2], bb[(2 * iw + 1) * 2 + 1]);
                        }
                    }
#pragma unroll
                    for (int half = 0; half < 2; half++) {
                        // sub-block j = 4*half + t of this block, rows g and g+8
                        uint32_t sc0, mm0, sc1, mm1;
                        if (half == 0) {
                            sc0 = x0 & 63u, mm0 = y0 & 63u, sc1 = x1 & 63u, mm1 = y1 & 63u;
                        } else {
                            sc0 = (z0 & 15u) | ((x0 >> 2) & 48u), mm0 = ((z0 >> 4) & 15u) | ((y0 >> 2) & 48u);
                            sc1 = (z1 & 15u) | ((x1 >> 2) & 48u), mm1 = ((z1 >> 4) & 15u) | ((y1 >> 2) & 48u);
                        }
                        const float fb = fbb[half * 4], sx = sxb[half * 4];
                        const float S0 =
                            ((dacc[half][0][0] + dacc[half][1][0]) + (dacc[half][0][1] + dacc[half][1][1])) * fb;
                        const float S1 =
                            ((dacc[half][0][2] + dacc[half][1][2]) + (dacc[half][0][3] + dacc[half][1][3])) * fb;
                        acc0 += (dn0.x * __uint2float_rn(sc0)) * S0 - (dn0.y * __uint2float_rn(mm0)) * sx;
                        acc1 += (dn1.x * __uint2float_rn(sc1)) * S1 - (dn1.y * __uint2float_rn(mm1)) * sx;
                    }
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
