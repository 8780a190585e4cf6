// tc_mmv.cuh -- decode matvec y = W.x for the quantized formats on sm_100a
// tensor cores: a TMA weight stream through an mbarrier ring, dequantisation in
// registers straight into MMA fragments, and a deterministic stream-K split.
// The per-format arithmetic lives in tc_q4k.cuh (Q4_K) and tc_q6k.cuh (Q6_K,
// repacked); this file is the machinery they share.
//
// Work split ("stream-K", deterministic).  Rows are taken 16 at a time (a
// "group", the MMA's M); a stage is (group, F::SBLK consecutive blocks).  The
// stages of all matrices of a batch, group-major, are split into one contiguous
// range per CTA (row_strip), so every SM gets the same number of bytes whatever
// the shapes.  A group cut by a CTA boundary is finished by whichever CTA
// arrives last at its counter, summing the pieces in CTA order; no spinning.
//
// Per CTA: warp 0 is the producer -- one 2-D TMA tensor copy per stage (a
// 16-row box of F::BOXW u64 of the weight matrix; rows past the end and columns
// past a row's end are zero-filled by the TMA unit; each CTA loads only its own tiles) into a ring
// of F::NSLOT slots, issued before griddepcontrol.wait so the stream overlaps
// the previous kernel under programmatic dependent launch.  F::NCW consumer
// warps form F::NSTREAM teams of F::NCONS; team j takes the CTA-local stages
// k = j (mod NSTREAM), and within a team warp w takes block w of the stage.  A warp copies its
// block's bytes to registers and releases the slot before any math.  Every
// mbarrier wait is bounded and reports through the device error word.
//
// One launch serves a batch of independent matvecs (the reference's
// matvec_lote, crates/soso-llm-core/src/gpu.rs:694-701: several matvecs, one
// wait); their stages are numbered one after another, so the batch streams as one.
#pragma once
#ifndef SB_GROUP_SLACK
#define SB_GROUP_SLACK 8  // stages a busiest CTA may take beyond the even split to avoid cut groups (build-time knob)
#endif
#include <cstring>

#include "tc_q4k.cuh"
#include "tc_q6k.cuh"
#include "tc_q80.cuh"
#include "group.cuh"

namespace sb {
namespace tcmv {

constexpr int MAXB = 40;           // matrices per launch
constexpr int CNT_MAX = 1 << 16;   // groups of 16 rows per launch (counters in the workspace)

struct __align__(64) MatDesc {
    CUtensorMap map;          // weights as [rows][row_bytes/8] u64, box 16 x F::BOXW
    const CUtensorMap *mapp;  // when set: the map to use instead (a table entry chosen on the device)
    const float *x;
    const float *xb;          // XS_SWIGLU: this matrix's b (else the batch's)
    float *y;
    int rows, cols, spg;    // spg: stages per 16-row group
    int st_begin, cnt_off;  // first global stage; first counter of its groups
    int pub_off;            // where this matrix's rows go in the batch's exchange slots (floats)
    int pairs;              // 1: rows are 16-row groups of gate and up in turn; y[i] = silu(gate_i) * up_i
};

constexpr int MAXGRID = 160;       // CTAs per launch at most (the per-CTA table)

// A batch as every CTA reads it: the header and this CTA's entry of the per-CTA table
// come first (a few cache lines, no dependent lookups before the weight stream starts),
// then the matrices.
struct Batch {
    int n, total;              // matrices, stages
    int max_cols, max_groups;  // shared-memory capacities (prep, partial table)
    int split_groups;          // 1: CTAs take whole 16-row groups (no cut groups, no fix-up)
    int pair_split;            // 1: ... two groups at a time (a matrix of gate/up group pairs)
    int total_groups;
    XSrc xs;                   // how every matrix's x is formed (tc_common.cuh)
    grp::Pub pub;              // also store every matrix's rows into the group's exchange areas
    grp::Wait wait;            // wait for an exchange point before reading the input
    int4 cta[MAXGRID];         // per CTA: first stage, end stage, first and last matrix touched
    MatDesc d[MAXB];
};

// Shared memory of the consumers besides the ring.
struct Work {
    uint8_t *prep;  // the prepared x of the current segment
    uint8_t *zero;  // 64 B of zeros
    float *part;    // [groups of this CTA][NCW][16]
    float *red;     // [64]
};

template <class F>
struct Smem {
    uint8_t *ring;    // NSLOT * SLOTB
    uint8_t *prep;    // F::prep_bytes(max_cols)
    uint8_t *zero;    // 64 B of zeros: the B fragment of lanes that carry no x
    float *part;      // [groups of this CTA][NCW][16]
    float *red;       // [64]: the sum of squares of an XS_NORM input, per unit or per consumer warp
    uint64_t *full;   // [NSLOT]
    uint64_t *empty;  // [NSLOT]
    __device__ Work work() const { return Work{prep, zero, part, red}; }
};

template <class F>
__host__ __device__ inline size_t smem_bytes(int max_cols, int max_groups)
{
    return (size_t)F::NSLOT * F::SLOTB + F::prep_bytes(max_cols) + 64 + (size_t)max_groups * F::NCW * 64 + 256 +
           2 * F::NSLOT * 8 + 64;
}

template <class F>
__device__ __forceinline__ Smem<F> carve(uint8_t *base, int max_cols, int max_groups)
{
    Smem<F> s;
    size_t o = 0;
    s.ring = base;
    o += (size_t)F::NSLOT * F::SLOTB;
    s.prep = base + o;
    o += F::prep_bytes(max_cols);
    s.zero = base + o;
    o += 64;
    s.part = reinterpret_cast<float *>(base + o);
    o += (size_t)max_groups * F::NCW * 64;
    s.red = reinterpret_cast<float *>(base + o);
    o += 256;
    o = (o + 7) & ~(size_t)7;
    s.full = reinterpret_cast<uint64_t *>(base + o);
    s.empty = s.full + F::NSLOT;
    return s;
}

// inverse of row_strip: which of n parts holds `unit`
__device__ __forceinline__ int owner_of(int unit, int total, int n)
{
    const int base = total / n, rem = total - base * n;
    const int big = rem * (base + 1);
    return unit < big ? unit / (base + 1) : rem + (base ? (unit - big) / base : 0);
}

// x of one segment -> the prepared fragments (s.prep), by the NCW consumer warps (named
// barrier 1).  Warp w takes units w, w + NCW, ...; the x values of PREP_U of its units are
// loaded before any of them is used, so one memory round trip serves them all.  XS_NORM
// (rmsnorm of h = a + b, or a + the weighted set): when every unit fits one such round, the
// sum of squares comes from the same loads -- per warp over its units, then over the warps
// in order -- and h, w are used from registers; wider inputs take a first pass for the sum.
// h_out (CTA 0 only): the new residual stream, each element stored once.  Every CTA reads
// the same x: each starts at a different unit (a rotation by its index), so that at any
// moment the CTAs ask the L2 for different lines instead of all for the same ones.
#ifndef SB_PREP_U
#define SB_PREP_U 2  // units per warp per load round (build-time tuning knob)
#endif
constexpr int PREP_U = SB_PREP_U;

template <class F>
__device__ __forceinline__ void prep_segment(XLoad &X, int cols, float *h_out, float eps, const Work &s, int cwg,
                                             int lane)
{
    constexpr int NCW = F::NCW, XPL = F::XPL;
    const int nu = F::units(cols), nv4 = cols / 4;
    const int rot = (int)((blockIdx.x * 5u) % (unsigned)nu);  // unit u -> slot (u + rot) % nu
    auto unit = [&](int q) { return q < nu ? (q + rot < nu ? q + rot : q + rot - nu) : nu; };
    const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float4 *ho = reinterpret_cast<float4 *>(h_out);
    if (X.mode == XS_NORM && nu <= PREP_U * NCW) {
        float4 v[PREP_U][XPL], w[PREP_U][XPL];
#pragma unroll
        for (int j = 0; j < PREP_U; j++)
#pragma unroll
            for (int k = 0; k < XPL; k++) {
                const int u = unit(cwg + j * NCW), i = F::xidx(u, lane, k);
                const bool in = u < nu && i < nv4;
                v[j][k] = in ? X.h(i) : zero;
                w[j][k] = in ? X.w[i] : zero;
            }
        // sum of squares per unit (lanes in a fixed order), then over the units in order: the
        // same in every CTA whatever the rotation
#pragma unroll
        for (int j = 0; j < PREP_U; j++) {
            const int u = unit(cwg + j * NCW);
            float ss = 0.0f;
#pragma unroll
            for (int k = 0; k < XPL; k++) {
                const float4 h = v[j][k];
                ss += (h.x * h.x + h.y * h.y) + (h.z * h.z + h.w * h.w);
                const int i = F::xidx(u, lane, k);
                if (ho && u < nu && i < nv4) ho[i] = h;
            }
            ss = warp_sum(ss);
            if (lane == 0 && u < nu) s.red[u] = ss;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
        float tot = 0.0f;
        for (int q = 0; q < nu; q++) tot += s.red[q];
        const float scale = 1.0f / sqrtf(tot / (float)cols + eps);
#pragma unroll
        for (int j = 0; j < PREP_U; j++) {
            const int u = unit(cwg + j * NCW);
            if (u >= nu) break;
#pragma unroll
            for (int k = 0; k < XPL; k++) {
                const float4 h = v[j][k], g = w[j][k];
                v[j][k] = make_float4(h.x * scale * g.x, h.y * scale * g.y, h.z * scale * g.z, h.w * scale * g.w);
            }
            F::prep_unit(u, nu, v[j], s.prep);
        }
        return;
    }
    if (X.mode == XS_NORM) {
        // sum of squares of h = a (+ b or the weighted residuals) first, in a fixed order
        float ss = 0.0f;
        for (int i = cwg * 32 + lane; i < nv4; i += NCW * 32) {
            const float4 v = X.h(i);
            if (ho) ho[i] = v;
            ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
        }
        ss = warp_sum(ss);
        if (lane == 0) s.red[cwg] = ss;
        asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
        float tot = 0.0f;
        for (int q = 0; q < NCW; q++) tot += s.red[q];
        X.scale = 1.0f / sqrtf(tot / (float)cols + eps);
    }
    for (int u0 = cwg; u0 < nu; u0 += PREP_U * NCW) {
        float4 v[PREP_U][XPL];
#pragma unroll
        for (int j = 0; j < PREP_U; j++)
#pragma unroll
            for (int k = 0; k < XPL; k++) {
                const int u = unit(u0 + j * NCW), i = F::xidx(u, lane, k);
                v[j][k] = u < nu && i < nv4 ? X(i) : zero;
            }
#pragma unroll
        for (int j = 0; j < PREP_U; j++) {
            const int u = unit(u0 + j * NCW);
            if (u >= nu) break;
            F::prep_unit(u, nu, v[j], s.prep);
        }
    }
}

// One format's ring of weight stages: NS slots of F::SLOTB bytes, a full barrier (the
// producer's TMA completion) and an empty barrier (the consumer team's release) per slot.
struct Ring {
    uint8_t *slot;
    uint64_t *full, *empty;
};

// The producer (one thread): TMA copies of this CTA's nst stages of batch B (its range
// starts at global stage st0, in matrix m_first) into ring r, stage k into slot k % NS;
// stage k >= NS first waits for the release of stage k - NS.  Returns the number of
// stages copied: nst, or fewer if a wait ran out.
template <class F, int NS>
__device__ __forceinline__ int produce(const Batch &B, const Ring &r, int st0, int m_first, int nst, uint64_t pol)
{
    int mi = m_first, slot = 0;
    unsigned phase = 0;  // parity of the empty-barrier phase to wait for
    const MatDesc *d = &B.d[mi];
    const CUtensorMap *mp = d->mapp ? d->mapp : &d->map;
    int G = (st0 - d->st_begin) / d->spg, j = (st0 - d->st_begin) - G * d->spg;
    int mend = d->st_begin + d->spg * ((d->rows + 15) >> 4);
    asm volatile("prefetch.tensormap [%0];" ::"l"(mp) : "memory");
    for (int k = 0; k < nst; k++) {
        if (st0 + k == mend) {  // next matrix of the batch
            d = &B.d[++mi];
            mp = d->mapp ? d->mapp : &d->map;
            G = 0, j = 0;
            mend = d->st_begin + d->spg * ((d->rows + 15) >> 4);
            asm volatile("prefetch.tensormap [%0];" ::"l"(mp) : "memory");
        }
        if (k >= NS && !mbar_wait(&r.empty[slot], phase)) return k;
        mbar_expect_tx_arrive(&r.full[slot], (unsigned)F::SLOTB);  // full box, zero-filled past the ends
        tma_load_2d(r.slot + slot * F::SLOTB, mp, F::stage_x(j), G * 16, &r.full[slot], pol);
        if (++j == d->spg) j = 0, G++;
        if (++slot == NS) {
            slot = 0;
            if (k >= NS) phase ^= 1u;  // stages 2*NS.. wait for the second use of a slot, ...
        }
    }
    return nst;
}

// Wait (bounded) until the TMA copies of the last issued stages, max(0, n - NS)..n-1, have
// landed: a CTA that gives up must not leave while copies into its shared memory are in flight.
template <int NS>
__device__ __forceinline__ void drain(const Ring &r, int n)
{
    for (int k = n > NS ? n - NS : 0; k < n; k++) mbar_wait(&r.full[k % NS], (unsigned)(k / NS) & 1u);
}

// The consumers of batch B (warp cwg of F::NCW, named barrier 1 among them): this CTA's
// stages (cr: first stage, end stage, first and last matrix) from ring r, every segment's
// x prepared first, rows written in the segment epilogue (cut groups' pieces to ws).
template <class F, int NS>
__device__ __forceinline__ void consume(const Batch &B, const Ring &r, const Work &s, Ws ws, int4 cr, int cwg,
                                        int lane, bool &failed)
{
    constexpr int NCW = F::NCW, NSTREAM = F::NSTREAM;
    static_assert(NS % NSTREAM == 0, "a ring slot must belong to one consumer team");
    const int st0 = cr.x, st1 = cr.y, m_first = cr.z, m_last = cr.w;
    const int nst = st1 - st0;
    const int team = cwg / F::NCONS, cw = cwg % F::NCONS, g = lane >> 2, t = lane & 3;
    const typename F::Lane L = F::lane_setup(g, t);
    {
        // this CTA's first matrix descriptor into the constant cache while the previous
        // kernel finishes (the asm keeps the load before the wait)
        const float *x_first = nst > 0 ? B.d[m_first].x : nullptr;
        asm volatile("" ::"l"(x_first));
    }
    griddep_wait();  // x of every matrix is written by the previous kernel
    if (B.wait.n) {  // the input's residual set comes from every rank of the group
        if (cwg == 0 && lane == 0)
            if (!grp::wait_counts(B.wait.cnt, B.wait.n, *B.wait.epoch * (unsigned)B.wait.per)) failed = true;
        asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
    }
    const float *prev_x = nullptr;
    int prev_cols = 0;
    for (int mi = m_first; mi <= m_last && nst > 0; mi++) {
        const MatDesc &d = B.d[mi];
        const int nb = F::units(d.cols), spg = d.spg;
        const int mtot = spg * ((d.rows + 15) >> 4);
        const int ka = max(st0, d.st_begin) - st0, kb = min(st1, d.st_begin + mtot) - st0;  // CTA-local stages
        const int gs0 = (ka + st0 - d.st_begin) / spg, gs1 = (kb - 1 + st0 - d.st_begin) / spg;
        const int ng = gs1 - gs0 + 1;
        // x -> prep (unless the previous segment prepared the same x) and a clean
        // partial table for this segment
        if (d.x != prev_x || d.cols != prev_cols) {
            XLoad X;
            X.a = reinterpret_cast<const float4 *>(d.x);
            X.b = reinterpret_cast<const float4 *>(d.xb ? d.xb : B.xs.b);
            X.w = reinterpret_cast<const float4 *>(B.xs.w);
            X.ys = reinterpret_cast<const float4 *>(B.xs.ys);
            X.scale = 1.0f;
            X.mode = B.xs.mode;
            X.ny = B.xs.mode == XS_NORM ? B.xs.ny : 0;
            X.ys4 = B.xs.ystride / 4;
            for (int k = 0; k < X.ny; k++) X.yw[k] = B.xs.yw[k];
            prep_segment<F>(X, d.cols, blockIdx.x == 0 ? B.xs.h_out : nullptr, B.xs.eps, s, cwg, lane);
            prev_x = d.x;
            prev_cols = d.cols;
        }
        for (int i = cwg * 32 + lane; i < ng * NCW * 16; i += NCW * 32) s.part[i] = 0.0f;
        asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
        const typename F::Seg S = F::seg_setup(L, s.prep, s.zero, nb, d.cols);
        float acc0 = 0.0f, acc1 = 0.0f;
        int cur = -1;
        // Team j takes the CTA-local stages k with k % NSTREAM == j in every segment, so
        // (NS a multiple of NSTREAM) each ring slot is only ever read by one team.  That
        // team waited for the slot's previous phase itself, so a parity wait can never
        // mistake the phase before an unfinished one for the awaited phase.
        const int k0 = ka + (team - ka % NSTREAM + NSTREAM) % NSTREAM;
        int slot = k0 % NS, G = (k0 + st0 - d.st_begin) / spg, j = (k0 + st0 - d.st_begin) - G * spg;
        unsigned parity = (k0 / NS) & 1;
        auto flush = [&]() {
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
            if (t == 0) {
                float *p = s.part + ((cur - gs0) * NCW + cwg) * 16;
                p[g] = acc0;
                p[g + 8] = acc1;
            }
        };
        for (int k = k0; k < kb && !failed; k += NSTREAM) {
            if (k != k0) {  // advance by NSTREAM stages
                slot += NSTREAM;
                if (slot >= NS) slot -= NS, parity ^= 1u;
                j += NSTREAM;
                while (j >= spg) j -= spg, G++;
            }
            if (!mbar_wait(&r.full[slot], parity)) {
                failed = true;
                set_dev_error(0x52u);
                break;
            }
            if (G != cur) {
                if (cur >= 0) flush();
                cur = G;
                acc0 = acc1 = 0.0f;
            }
            const int blk = j * F::SBLK + cw;
            if (blk < nb) {
                F::block(L, S, r.slot + slot * F::SLOTB, cw, blk, nb, &r.empty[slot], acc0, acc1);
            } else {
                __syncwarp();
                if (lane == 0) mbar_arrive(&r.empty[slot]);
            }
        }
        if (cur >= 0) flush();
        asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
        // segment epilogue: sum the consumer warps' pieces per group (fixed order)
        const bool head_cut = mi == m_first && (st0 - d.st_begin) % spg != 0;
        const bool tail_cut = mi == m_last && (st1 - d.st_begin) % spg != 0 && st1 < d.st_begin + mtot;
        if (d.pairs) {
            // gate/up group pairs (whole in this CTA): y = silu(gate) * up (gemm.rs:210-226,
            // the same f32 steps as the XS_SWIGLU input form)
            for (int i = cwg * 32 + lane; i < (ng >> 1) * 16; i += NCW * 32) {
                const int pl = i >> 4, rr = i & 15, row = ((gs0 >> 1) + pl) * 16 + rr;
                float vg = 0.0f, vu = 0.0f;
                for (int w = 0; w < NCW; w++) {
                    vg += s.part[(2 * pl * NCW + w) * 16 + rr];
                    vu += s.part[((2 * pl + 1) * NCW + w) * 16 + rr];
                }
                if (2 * row < d.rows) d.y[row] = vg / (1.0f + expf(-vg)) * vu;
            }
            asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
            continue;
        }
        for (int i = cwg * 32 + lane; i < ng * 16; i += NCW * 32) {
            const int gl = i >> 4, rr = i & 15, row = (gs0 + gl) * 16 + rr;
            float v = 0.0f;
            for (int w = 0; w < NCW; w++) v += s.part[(gl * NCW + w) * 16 + rr];
            const bool cut = (gl == 0 && head_cut) || (gl == ng - 1 && tail_cut);
            if (!cut) {
                if (row < d.rows) {
                    d.y[row] = v;
                    for (int p = 0; p < B.pub.n; p++) B.pub.dst[p][d.pub_off + row] = v;
                }
            } else {
                // side 0: the group holding this CTA's first stage, side 1: any other (its last)
                const int ga = d.st_begin + (gs0 + gl) * spg;
                ws.part[(blockIdx.x * 2 + ((st0 >= ga && st0 < ga + spg) ? 0 : 1)) * 16 + rr] = v;
                __threadfence();
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
    }
}

// Every row this CTA owns is in the peers' exchange areas: count the CTA there (all CTAs
// count, so the consumers' target is epoch * grid whatever the split).  All threads.
__device__ __forceinline__ void publish_count(const Batch &B)
{
    if (B.pub.n) {
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x < B.pub.n) atomicAdd_system(B.pub.cnt[threadIdx.x], 1u);
    }
}

template <class F, bool DEV>
__device__ __forceinline__ void tc_mmv_body(const Batch &B, Ws ws)
{
    // A batch in device memory may have been written by the previous kernel (the expert
    // choice): everyone, the producer included, waits for it before reading the batch.
    if (DEV) griddep_wait();
    constexpr int NSLOT = F::NSLOT;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Smem<F> s = carve<F>(smem_raw, B.max_cols, B.max_groups);
    const Ring ring{s.ring, s.full, s.empty};
    const int4 cr = B.cta[blockIdx.x];  // (built on the host: fill_cta)
    const int st0 = cr.x, st1 = cr.y, m_first = cr.z, m_last = cr.w;
    const int nst = st1 - st0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int k = 0; k < NSLOT; k++) {
            mbar_init(&s.full[k], 1);
            mbar_init(&s.empty[k], F::NCONS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < 16) reinterpret_cast<float *>(s.zero)[threadIdx.x] = 0.0f;
    __syncthreads();
    // Dependents may launch now: they only read what this grid writes after their
    // own griddepcontrol.wait, which waits for this grid to complete.
    griddep_launch();

    bool failed = false;
    int issued = 0;
    if (warp == 0) {
        // ---------------- producer: weights do not depend on the previous kernel, so the
        // whole stream runs without griddepcontrol.wait
        if (lane == 0 && nst > 0) {
            issued = produce<F, NSLOT>(B, ring, st0, m_first, nst, l2_evict_first());
            if (issued < nst) {
                failed = true;
                set_dev_error(0x51u);
            }
        }
        __syncwarp();
    } else {
        consume<F, NSLOT>(B, ring, s.work(), ws, cr, warp - 1, lane, failed);
    }
    // let every TMA copy issued into this CTA's shared memory land before exiting (bounded)
    if (failed && warp == 0 && lane == 0) drain<NSLOT>(ring, issued);
    publish_count(B);
    if (B.split_groups) return;  // whole groups: every row is final in the CTA that formed it
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
                const int cs0 = B.cta[c].x;
                // CTA c stored G as side 0 if its range starts inside G, else as side 1
                v += __ldcg(&ws.part[(c * 2 + ((cs0 >= ga && cs0 < ge) ? 0 : 1)) * 16 + r]);
            }
            if (G * 16 + r < d.rows) d.y[G * 16 + r] = v;
            if (r == 0) ws.cnt[d.cnt_off + G] = 0u;
        }
    }
}

template <class F>
__global__ void __launch_bounds__(F::THREADS, F::MINB) tc_mmv_kernel(const __grid_constant__ Batch B, Ws ws)
{
    tc_mmv_body<F, false>(B, ws);
}

// The same with the batch in device memory (written by an earlier kernel on the stream,
// e.g. the expert choice of a MoE router); its matrices name their maps through mapp.
// With `sel` set, the batch is B[*sel], one of several prepared batches (the number of
// routed experts this rank owns picks the one whose split fits).
template <class F>
__global__ void __launch_bounds__(F::THREADS, F::MINB) tc_mmv_dev_kernel(const Batch *__restrict__ B,
                                                                   const int *__restrict__ sel, Ws ws)
{
    if (sel) {
        griddep_wait();  // *sel is written by the previous kernel
        tc_mmv_body<F, true>(B[*sel], ws);
    } else {
        tc_mmv_body<F, true>(*B, ws);
    }
}

// ------------------------------------------------------------------ host side

// Workspace layout (fixed offsets, whatever the shape, because one workspace
// serves every launch on a stream): [cnt: CNT_MAX u32, zero between launches]
// [part: grid*2*16 f32].  Zeroed once when allocated; the kernel leaves it zeroed.
inline size_t ws_part_off() { return (size_t)CNT_MAX * 4; }
inline size_t ws_bytes(int grid) { return ws_part_off() + (size_t)grid * 2 * 16 * 4 + 256; }
inline Ws ws_of(void *p)
{
    uint8_t *b = reinterpret_cast<uint8_t *>(p);
    Ws w;
    w.cnt = reinterpret_cast<unsigned *>(b);
    w.part = reinterpret_cast<float *>(b + ws_part_off());
    return w;
}

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

// Weights as a [rows][row_bytes/8] u64 tensor, box = 16 rows x F::BOXW u64.
template <class F>
inline int make_map(CUtensorMap *m, const void *w, int rows, int cols)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) return -6;
    const cuuint64_t rb = (cuuint64_t)F::row_bytes(cols);
    cuuint64_t dims[2] = {rb / 8, (cuuint64_t)rows};
    cuuint64_t strides[1] = {rb};
    cuuint32_t box[2] = {(cuuint32_t)F::BOXW, 16};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(w), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -7;
}

// Tensor maps are pure functions of (format, pointer, shape); keep the last few.
template <class F>
inline int cached_map(CUtensorMap *out, const void *w, int rows, int cols)
{
    struct E {
        const void *w;
        int rows, cols;
        CUtensorMap m;
    };
    static E cache[128];
    static int next = 0;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    for (auto &e : cache)
        if (e.w == w && e.rows == rows && e.cols == cols) {
            *out = e.m;
            return 0;
        }
    E &e = cache[next];
    next = (next + 1) % 128;
    const int rc = make_map<F>(&e.m, w, rows, cols);
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

template <class F>
inline int stages_per_group(int cols)
{
    return (F::units(cols) + F::SBLK - 1) / F::SBLK;
}

// Shared memory for a batch over `grid` CTAs.
template <class F>
inline size_t batch_smem(const MatOp *ops, int n, int grid, int *max_cols, int *max_groups)
{
    long long total = 0;
    int mc = 0;
    for (int i = 0; i < n; i++) {
        total += (long long)stages_per_group<F>(ops[i].cols) * ((ops[i].rows + 15) / 16);
        mc = ops[i].cols > mc ? ops[i].cols : mc;
    }
    const long long per = (total + grid - 1) / grid;
    int mg = 1;
    for (int i = 0; i < n; i++) {
        const int spg = stages_per_group<F>(ops[i].cols), groups = (ops[i].rows + 15) / 16;
        const long long g = per / spg + 2;
        const int gi = (int)(g < groups ? g : groups);
        mg = gi > mg ? gi : mg;
    }
    *max_cols = mc;
    *max_groups = mg;
    return smem_bytes<F>(mc, mg);
}

template <class F>
inline bool fits(const MatOp *ops, int n, int grid)
{
    int mc, mg;
    for (int i = 0; i < n; i++)
        if (ops[i].cols > F::MAX_COLS || ops[i].cols % F::COLS_MULT || ops[i].rows < 1) return false;
    return batch_smem<F>(ops, n, grid, &mc, &mg) <= 227 * 1024;
}

// Launch a batch of up to MAXB independent matvecs of format F on `stream`, with
// the scratch given as counter / partial pointers (counters zero on entry, left
// zero); at most cnt_cap 16-row groups in the batch.
// Stages of the busiest CTA when whole groups are split evenly over `grid` CTAs.
inline int group_split_max(const Batch &b, int grid)
{
    int mx = 0;
    auto stage_of = [&](int g) {
        if (g >= b.total_groups) return b.total;
        int i = 0;
        while (i + 1 < b.n && b.d[i + 1].cnt_off <= g) i++;
        return b.d[i].st_begin + (g - b.d[i].cnt_off) * b.d[i].spg;
    };
    for (int c = 0; c < grid; c++) {
        const int base = b.total_groups / grid, rem = b.total_groups % grid;
        const int g0 = c * base + (c < rem ? c : rem), g1 = g0 + base + (c < rem ? 1 : 0);
        const int st = stage_of(g1) - stage_of(g0);
        mx = st > mx ? st : mx;
    }
    return mx;
}

struct MatOpX {  // a MatOp with a per-matrix second input (XS_SWIGLU) and an optional map table entry
    MatOp op;
    const float *xb;
    const CUtensorMap *mapp;
    int pairs = 0;   // gate/up group pairs: y has rows / 2 entries (MatDesc::pairs)
};

// The per-CTA table of a batch over `grid` CTAs: each CTA's stage range (whole groups or an
// even stage split, as split_groups says) and the matrices it touches.
inline int fill_cta(Batch *b, int grid)
{
    if (grid < 1 || grid > MAXGRID) return -1;
    auto stage_of = [&](int g) {
        if (g >= b->total_groups) return b->total;
        int i = 0;
        while (i + 1 < b->n && b->d[i + 1].cnt_off <= g) i++;
        return b->d[i].st_begin + (g - b->d[i].cnt_off) * b->d[i].spg;
    };
    for (int c = 0; c < grid; c++) {
        int st0, st1;
        if (b->split_groups) {
            int g0, g1;
            if (b->pair_split) {
                row_strip(b->total_groups / 2, c, grid, g0, g1);
                g0 *= 2, g1 *= 2;
            } else {
                row_strip(b->total_groups, c, grid, g0, g1);
            }
            st0 = stage_of(g0), st1 = stage_of(g1);
        } else {
            row_strip(b->total, c, grid, st0, st1);
        }
        int mf = 0;
        while (mf + 1 < b->n && b->d[mf + 1].st_begin <= st0) mf++;
        int ml = mf;
        while (st1 > st0 && ml + 1 < b->n && b->d[ml + 1].st_begin < st1) ml++;
        b->cta[c] = make_int4(st0, st1, mf, ml);
    }
    return 0;
}

// Fill *b (every field) for n matrices over `grid` CTAs; *smem = its dynamic shared memory.
// With `uniform_x` false the matrices may have different inputs (XS_PLAIN / XS_SWIGLU).
template <class F>
inline int build_batch(const MatOpX *ops, int n, int cnt_cap, int grid, const XSrc *xs, Batch *bp, size_t *smem_out)
{
    if (n < 1 || n > MAXB) return -1;
    Batch &b = *bp;
    int st = 0, cnt = 0;
    MatOp plain[MAXB];
    for (int i = 0; i < n; i++) {
        const MatOp &o = ops[i].op;
        plain[i] = o;
        if (o.cols > F::MAX_COLS || o.cols % F::COLS_MULT || o.rows < 1) return -1;
        MatDesc &d = b.d[i];
        const int mrc = cached_map<F>(&d.map, o.w, o.rows, o.cols);
        if (mrc) return mrc;
        d.mapp = ops[i].mapp;
        d.x = o.x;
        d.xb = ops[i].xb;
        d.y = o.y;
        d.rows = o.rows;
        d.cols = o.cols;
        d.spg = stages_per_group<F>(o.cols);
        d.st_begin = st;
        d.cnt_off = cnt;
        d.pub_off = 0;
        d.pairs = ops[i].pairs;
        if (ops[i].pairs != ops[0].pairs || (d.pairs && o.rows % 32)) return -1;  // all pair matrices or none
        st += d.spg * ((o.rows + 15) / 16);
        cnt += (o.rows + 15) / 16;
    }
    if (cnt > cnt_cap) return -1;
    b.n = n;
    b.total = st;
    b.total_groups = cnt;
    b.xs = xs ? *xs : XSrc{};
    b.pub = grp::Pub{};
    b.wait = grp::Wait{};
    if (b.xs.mode != XS_PLAIN) {
        if (b.xs.mode != XS_NORM && b.xs.mode != XS_SWIGLU) return -1;
        if (b.xs.mode == XS_NORM) {
            // one input vector for the whole batch (h_out is written once, from it)
            for (int i = 1; i < n; i++)
                if (ops[i].op.x != ops[0].op.x || ops[i].op.cols != ops[0].op.cols) return -1;
            if (!b.xs.w || b.xs.ny < 0 || b.xs.ny > XS_MAXY || (b.xs.ny && (!b.xs.ys || !b.xs.yw))) return -1;
            if (b.xs.ny && b.xs.ystride % 4) return -2;
        } else {
            for (int i = 0; i < n; i++)
                if (!ops[i].xb && !b.xs.b) return -1;
        }
        if (((uintptr_t)b.xs.b | (uintptr_t)b.xs.w | (uintptr_t)b.xs.h_out | (uintptr_t)b.xs.ys) & 15) return -2;
    }
    for (int i = 0; i < n; i++)
        if ((uintptr_t)ops[i].xb & 15) return -2;
    // Whole groups per CTA when that costs at most one stage more on the busiest CTA
    // and the stream-K split is short (latency-bound), or at most SB_GROUP_SLACK stages more
    // (a stage streams in well under the cross-CTA fix-up's round trip): no fix-up at all.
    const int smax = (st + grid - 1) / grid, gmax = group_split_max(b, grid);
    b.split_groups = gmax <= smax || (gmax <= smax + 1 && smax <= 4) || gmax <= smax + SB_GROUP_SLACK;
    b.pair_split = ops[0].pairs;
    if (b.pair_split) b.split_groups = 1;  // a pair's two groups finish in one CTA
    size_t smem = batch_smem<F>(plain, n, grid, &b.max_cols, &b.max_groups);
    if (b.split_groups) {
        const int need = b.pair_split ? 2 * ((cnt / 2 + grid - 1) / grid) + 2 : (cnt + grid - 1) / grid + 1;
        if (need > b.max_groups && smem_bytes<F>(b.max_cols, need) <= 227 * 1024) {
            b.max_groups = need;
            smem = smem_bytes<F>(b.max_cols, need);
        } else if (need > b.max_groups) {
            if (b.pair_split) return -5;
            b.split_groups = 0;
        }
    }
    if (smem > 227 * 1024) return -5;
    *smem_out = smem;
    return fill_cta(&b, grid);
}

// A published matrix's rows must be final in the CTA that computes them: switch a batch
// to whole 16-row groups per CTA (no groups cut between CTAs), growing *smem to match.
template <class F>
inline int whole_groups(Batch *b, int grid, size_t *smem)
{
    if (b->split_groups) return 0;
    const int need = (b->total_groups + grid - 1) / grid + 1;
    if (need > b->max_groups) b->max_groups = need;
    *smem = smem_bytes<F>(b->max_cols, b->max_groups);
    if (*smem > 227 * 1024) return -5;
    b->split_groups = 1;
    return fill_cta(b, grid);
}

// A batch of no matrices (every CTA only takes part in the publication, if any); *smem
// is what its launch needs at least.
template <class F>
inline void empty_batch(Batch *b, const XSrc &xs, size_t *smem)
{
    memset(b, 0, sizeof(Batch));
    b->xs = xs;
    b->split_groups = 1;
    b->max_groups = 1;
    *smem = smem_bytes<F>(0, 1);
}

// Raise a kernel's dynamic shared-memory limit to `smem` (only ever grows; one record per
// device and kernel).
template <class K>
inline int ensure_smem(K kernel, size_t smem, size_t *rec)
{
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return -3;
    if (smem > rec[dev]) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return -3;
        rec[dev] = smem;
    }
    return 0;
}

inline cudaLaunchConfig_t mmv_config(int grid, int threads, size_t smem, int pdl, cudaStream_t stream,
                                     cudaLaunchAttribute *attr)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

// Launch a batch of up to MAXB independent matvecs of format F on `stream`, with
// the scratch given as counter / partial pointers (counters zero on entry, left
// zero); at most cnt_cap 16-row groups in the batch.
template <class F>
inline int launch_batch_ws(const MatOp *ops, int n, Ws wsd, int cnt_cap, int grid, int pdl, cudaStream_t stream,
                           const XSrc *xs = nullptr, const grp::Pub *pub = nullptr, const grp::Wait *wait = nullptr,
                           bool pairs = false)
{
    if (n < 1 || n > MAXB) return -1;
    static Batch b;  // large: built host-side, passed by value as the kernel parameter
    static std::mutex mu;
    static size_t smem_rec[64];
    std::lock_guard<std::mutex> lk(mu);
    MatOpX ox[MAXB];
    for (int i = 0; i < n; i++) ox[i] = MatOpX{ops[i], nullptr, nullptr, pairs ? 1 : 0};
    size_t smem = 0;
    int rc = build_batch<F>(ox, n, cnt_cap, grid, xs, &b, &smem);
    if (rc) return rc;
    if (wait) b.wait = *wait;
    if (pub && pub->n) {
        if (n != 1) return -1;
        b.pub = *pub;
        if ((rc = whole_groups<F>(&b, grid, &smem))) return rc;
    }
    if ((rc = ensure_smem(tc_mmv_kernel<F>, smem, smem_rec))) return rc;
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = mmv_config(grid, F::THREADS, smem, pdl, stream, attr);
    return cudaLaunchKernelEx(&cfg, tc_mmv_kernel<F>, b, wsd) == cudaSuccess ? 0 : -4;
}

// Launch a batch held in device memory (dev, a copy of a batch made by build_batch, whose
// mapp / x / y / pub_off fields an earlier kernel on the stream may have rewritten; shapes
// and the split must stay as built), or dev[*sel] when sel is set.  smem: at least what
// build_batch returned for every batch that may be chosen.
template <class F>
inline int launch_dev_batch(const Batch *dev, const int *sel, size_t smem, Ws wsd, int grid, int pdl,
                            cudaStream_t stream)
{
    static size_t smem_rec[64];
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    int rc = ensure_smem(tc_mmv_dev_kernel<F>, smem, smem_rec);
    if (rc) return rc;
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = mmv_config(grid, F::THREADS, smem, pdl, stream, attr);
    return cudaLaunchKernelEx(&cfg, tc_mmv_dev_kernel<F>, dev, sel, wsd) == cudaSuccess ? 0 : -4;
}

// As launch_batch_ws over a workspace of ws_bytes(grid) bytes.
template <class F>
inline int launch_batch(const MatOp *ops, int n, void *ws, int grid, int pdl, cudaStream_t stream,
                        const XSrc *xs = nullptr, const grp::Pub *pub = nullptr, const grp::Wait *wait = nullptr,
                        bool pairs = false)
{
    return launch_batch_ws<F>(ops, n, ws_of(ws), CNT_MAX, grid, pdl, stream, xs, pub, wait, pairs);
}

// Repack GGML Q6_K rows (reference layout) into the packed layout of tc_q6k.cuh.
inline int q6k_pack(const void *src, size_t rows, size_t cols, void *dst, cudaStream_t stream)
{
    if (!src || !dst || !rows || cols % 256 || cols > (1u << 24) || rows > (1u << 30)) return -1;
    const long long nb = (long long)(cols / 256), n = (long long)rows * nb;
    const unsigned blocks = (unsigned)((n + 255) / 256);
    q6k_pack_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const uint8_t *>(src), (long long)rows, (int)nb,
                                                reinterpret_cast<uint8_t *>(dst),
                                                (long long)q6k_packed_row_bytes(cols));
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace tcmv
}  // namespace sb
