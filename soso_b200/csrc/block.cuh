// block.cuh -- the steps of a block prefill between the GEMMs (pgemm.cuh): n tokens at
// positions pos0 .. pos0 + n - 1 through one layer, as the reference's forward_layer_block
// (crates/soso-llm-core/src/layer.rs:1433) runs them.
//
//   norm16_rows      h = a (+ res), x = rmsnorm(h) * w (gemm.rs:93-100, add_f32 :265) into
//                    f16 GEMM operands (and f32 when a shared-expert gate needs it)
//   rope_kv_rows     bias, QK-norm, RoPE and the f16 K/V append of every token
//                    (layer.rs:1146-1193, kv.rs:258-275): the decode step's math per row
//   attn_prefill     causal GQA / MHA attention over the f16 rows on the tensor cores
//                    (attention_decode_f16_tiled_scalar, attn.rs:73-140, per query row;
//                    the reference's block kernels are attn_prefill_f16 and its mma form,
//                    lxdde/ports/nouveau/matvec_iq.cu:507-628, :1477+)
//   mla_*            the MLA latent rows (f16, kv.rs:293-315), RoPE of the q and the expanded
//                    k rope slices (llama pairs, gemm.rs:1346) and the rope-key cache
//   moe_*            routing of every token (topk_softmax, gemm.rs:62-91), grouping of the
//                    (token, choice) pairs by expert with the GEMM tile tables, the gather of
//                    their inputs, and the weighted combine in choice order
//                    (layer.rs:1922-1933, shared expert layer.rs:1883-1907)
#pragma once
#include "pgemm.cuh"

namespace sb {
namespace blk {

// ---- norm rows -------------------------------------------------------------------
// One CTA per token row: h = a (+ res) -> h_out (when set); x = rmsnorm(h) * w as f16 (x16)
// and f32 (x32, when set).  The sum of squares runs per thread over a fixed stride, then
// over the threads in order.
__global__ void norm16_rows_kernel(const float *__restrict__ a, const float *__restrict__ res, float *h_out,
                                   const float *__restrict__ w, __half *x16, float *x32, int n, float eps)
{
    __shared__ float red[32];
    griddep_wait();
    const size_t base = (size_t)blockIdx.x * n;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float h = a[base + i] + (res ? res[base + i] : 0.0f);
        ss += h * h;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int k = 0; k < (int)(blockDim.x >> 5); k++) tot += red[k];
    const float scale = 1.0f / sqrtf(tot / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float h = a[base + i] + (res ? res[base + i] : 0.0f);
        if (h_out) h_out[base + i] = h;
        const float x = h * scale * w[i];
        x16[base + i] = __float2half_rn(x);
        if (x32) x32[base + i] = x;
    }
    griddep_launch();
}

// out = a + b over count floats (a block's residual with its pending output).
__global__ void add_rows_kernel(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ out,
                                long long count)
{
    griddep_wait();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count; i += (long long)gridDim.x * blockDim.x)
        out[i] = a[i] + b[i];
    griddep_launch();
}

// f32 rows -> f16 rows (GEMM operands), 4 elements a thread.
__global__ void to16_kernel(const float *__restrict__ x, __half *__restrict__ y, long long total4)
{
    griddep_wait();
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total4;
         i += (long long)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(x)[i];
        reinterpret_cast<__half2 *>(y)[2 * i] = __floats2half2_rn(v.x, v.y);
        reinterpret_cast<__half2 *>(y)[2 * i + 1] = __floats2half2_rn(v.z, v.w);
    }
    griddep_launch();
}

// ---- GQA: bias, QK-norm, RoPE, K/V append of every token --------------------------
// grid (heads + 2 kv_heads, n), head_dim / 2 threads: the decode step's rope_kv_kernel
// (decode_ops.cuh) on row t of the stacked [q | k | v] rows at position pos0 + t.
struct RopeRowsArgs {
    float *qkv;  // [n][qd + 2 kvd]
    const float *bias, *qnorm, *knorm;
    uint16_t *kc, *vc;
    int pos0, heads, kv_heads, hd, ctx;
    float theta, eps;
    int neox;
    const float *factors;
    float mscale;
};

__global__ void rope_kv_rows_kernel(RopeRowsArgs a)
{
    __shared__ float red[32];
    griddep_wait();
    const int h = blockIdx.x, i = threadIdx.x, half = a.hd >> 1, t = blockIdx.y;
    const int kvd = a.kv_heads * a.hd, pos = a.pos0 + t;
    if (pos < 0 || pos >= a.ctx) {
        if (i == 0 && h == 0) set_dev_error(0x91u);
        return;
    }
    float *qkv = a.qkv + (size_t)t * (a.heads * a.hd + 2 * kvd);
    int base, kind;  // kind 0 = q, 1 = k, 2 = v
    if (h < a.heads) kind = 0, base = h * a.hd;
    else if (h < a.heads + a.kv_heads) kind = 1, base = a.heads * a.hd + (h - a.heads) * a.hd;
    else kind = 2, base = a.heads * a.hd + kvd + (h - a.heads - a.kv_heads) * a.hd;
    const int e0 = a.neox ? i : 2 * i, e1 = a.neox ? i + half : 2 * i + 1;
    float v0 = qkv[base + e0], v1 = qkv[base + e1];
    if (a.bias) {
        v0 += a.bias[base + e0];
        v1 += a.bias[base + e1];
    }
    const float *nw = kind == 0 ? a.qnorm : kind == 1 ? a.knorm : nullptr;
    if (nw) {
        float ss = v0 * v0 + v1 * v1;
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((i & 31) == 0) red[i >> 5] = ss;
        __syncthreads();
        float tot = 0.0f;
        for (int k = 0; k < (int)((blockDim.x + 31) >> 5); k++) tot += red[k];
        const float scale = 1.0f / sqrtf(tot / (float)a.hd + a.eps);
        v0 = v0 * scale * nw[e0];
        v1 = v1 * scale * nw[e1];
    }
    if (kind < 2) {
        float freq = powf(a.theta, (-2.0f * (float)i) / (float)a.hd);
        if (a.factors) freq /= a.factors[i];
        const float ang = (float)pos * freq;
        const float s = sinf(ang) * a.mscale, c = cosf(ang) * a.mscale;
        const float r0 = v0 * c - v1 * s, r1 = v0 * s + v1 * c;
        if (kind == 0) {
            qkv[base + e0] = r0;
            qkv[base + e1] = r1;
        } else {
            uint16_t *row = a.kc + (size_t)pos * kvd + (base - a.heads * a.hd);
            row[e0] = f32_to_f16_ref(r0);
            row[e1] = f32_to_f16_ref(r1);
        }
    } else {
        uint16_t *row = a.vc + (size_t)pos * kvd + (base - a.heads * a.hd - kvd);
        row[e0] = f32_to_f16_ref(v0);
        row[e1] = f32_to_f16_ref(v1);
    }
    griddep_launch();
}

// ---- causal attention of a block of queries --------------------------------------
// Query row (token t, head h) at position pos0 + t attends keys 0 .. pos0 + t of kv head
// h / (heads / kv_heads): softmax(q.k / sqrt(dqk)) . v per row (attention_decode_f16_tiled_scalar,
// attn.rs:73-140, over the f16 rows; the reference's block kernels are attn_prefill_f16 and its
// mma.sync form, lxdde/ports/nouveau/matvec_iq.cu:507-628, :1477+).  On the tensor cores
// (mma.sync m16n8k16, f32 accumulation): a CTA takes 64 query rows of one kv head (64 / G
// tokens x the G heads of the group), each of its 4 warps 16 rows; keys stream through shared
// memory 32 at a time (cp.async, two buffers).  S = Q K^T with q split into f16 hi + lo (22
// significant bits, as the decode attention; K and V are f16 already), the causal mask, an
// online softmax per row in f32 (running maximum and sum, the reference's order of
// operations per key block), O += P V with P in f16.
constexpr int AP_ROWS = 64, AP_KB = 32, AP_WARPS = 4, AP_MAXD = 256;

struct AttnPrefillArgs {
    const float *q;      // [n][heads][dqk] (row stride ldq floats)
    const uint16_t *k;   // key rows: key t, kv head g at k + t * ldk + g * dqk  (f16)
    const uint16_t *v;   // value rows: v + t * ldv + g * dv (f16)
    float *out;          // [n][heads][dv] (row stride ldo floats)
    int n, pos0, heads, kv_heads, dqk, dv, ldq, ldk, ldv, ldo;
    float scale;
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(tcmv::smem_u32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b)
{
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Shared memory of attn_prefill_kernel<KQ, NV, QS>: q hi / lo staging [2][64][QP] (kept for
// the whole kernel when QS, else reused) and the key / value double buffers [2][32][QP],
// [2][32][VP] (f16, row pitches padded by 16 bytes against bank conflicts).
template <int KQ, int NV, bool QS, int KS>
__host__ __device__ constexpr size_t attn_prefill_smem()
{
    constexpr size_t QP = 16 * KQ + 8, VP = 8 * NV + 8, qbytes = 2 * AP_ROWS * QP * 2,
                     kvbytes = 2 * KS * AP_KB * (QP + VP) * 2, merge = AP_ROWS * (8 * NV + 2) * 4;
    constexpr size_t a = QS ? qbytes + kvbytes : (qbytes > kvbytes ? qbytes : kvbytes);
    return a > merge ? a : merge;
}

// Widths up to 16 KQ (q, k) and 8 NV (v) that are multiples of 8: the columns past a.dqk /
// a.dv are zero in shared memory and drop out of both products.  QS: the q fragments are
// read from shared memory at every key block instead of being held in registers (the
// 256-wide heads, whose q hi / lo and output accumulators would not fit in registers).
// KS = 2: eight warps, the keys of each 64-key stage split between two groups of four (one
// online softmax each, merged at the end), so that twice the warps hide the MMA and load
// latencies of a CTA's 64 rows.
template <int KQ, int NV, bool QS, int KS>
__global__ void __launch_bounds__(KS *AP_WARPS * 32) attn_prefill_kernel(AttnPrefillArgs a)
{
    constexpr int DQ = 16 * KQ, DV = 8 * NV, QP = DQ + 8, VP = DV + 8;  // row pitches (f16)
    constexpr int NT = KS * AP_WARPS * 32, SKEYS = KS * AP_KB;         // threads, keys a stage
    extern __shared__ __align__(16) uint16_t ap_smem[];
    uint16_t *qh = ap_smem, *ql = qh + AP_ROWS * QP;                   // q hi / lo
    uint16_t *ks = QS ? ql + AP_ROWS * QP : ap_smem, *vs = ks + 2 * SKEYS * QP;
    griddep_wait();
    // the CTA's 64 rows: tpc tokens x the G query heads of kv head g (rows past tpc G idle)
    const int G = a.heads / a.kv_heads, g = blockIdx.y, tpc = AP_ROWS / G, t0 = blockIdx.x * tpc;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
    const int rw = warp % AP_WARPS, kh = warp / AP_WARPS;  // row group, key group
    // q of the CTA's rows -> f16 hi / lo in shared memory: 16-byte loads, a batch of them in
    // flight before the first is used
    {
        constexpr int C4 = DQ / 4, PER = AP_ROWS * C4 / NT;
        constexpr int NB = PER % 8 == 0 ? 8 : PER % 4 == 0 ? 4 : PER % 2 == 0 ? 2 : 1;
        static_assert(AP_ROWS * C4 % NT == 0 && PER % NB == 0, "q staging shape");
#pragma unroll 1
        for (int i0 = 0; i0 < PER; i0 += NB) {
            float4 xv[NB];
#pragma unroll
            for (int u = 0; u < NB; u++) {
                const int i = threadIdx.x + (i0 + u) * NT, r = i / C4, d = 4 * (i % C4);
                const int t = t0 + r / G, hh = g * G + r % G;
                xv[u] = r < tpc * G && t < a.n && d < a.dqk
                            ? *reinterpret_cast<const float4 *>(a.q + (size_t)t * a.ldq + hh * a.dqk + d)
                            : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < NB; u++) {
                const int i = threadIdx.x + (i0 + u) * NT, r = i / C4, d = 4 * (i % C4);
                uint16_t hi[4], lo[4];
                split_f16(xv[u].x, hi[0], lo[0]);
                split_f16(xv[u].y, hi[1], lo[1]);
                split_f16(xv[u].z, hi[2], lo[2]);
                split_f16(xv[u].w, hi[3], lo[3]);
                *reinterpret_cast<uint2 *>(qh + r * QP + d) =
                    make_uint2(hi[0] | ((uint32_t)hi[1] << 16), hi[2] | ((uint32_t)hi[3] << 16));
                *reinterpret_cast<uint2 *>(ql + r * QP + d) =
                    make_uint2(lo[0] | ((uint32_t)lo[1] << 16), lo[2] | ((uint32_t)lo[3] << 16));
            }
        }
    }
    __syncthreads();
    const int mi = lane >> 3, mr = lane & 7;
    const int qrow = 16 * rw + mr + (mi & 1) * 8, qcol = (mi >> 1) * 8;  // ldmatrix addresses
    uint32_t fqh[QS ? 1 : KQ][4], fql[QS ? 1 : KQ][4];
    if constexpr (!QS) {
#pragma unroll
        for (int s = 0; s < KQ; s++) {
            ldsm_x4(fqh[s], qh + qrow * QP + 16 * s + qcol);
            ldsm_x4(fql[s], ql + qrow * QP + 16 * s + qcol);
        }
        __syncthreads();  // the staging area becomes the key / value buffers
    }
    // this thread's two rows (gq, gq + 8 of the warp): their last key
    int lim[2];
#pragma unroll
    for (int h2 = 0; h2 < 2; h2++) {
        const int r = 16 * rw + gq + 8 * h2, t = t0 + r / G;
        lim[h2] = r < tpc * G && t < a.n ? a.pos0 + t : -1;
    }
    const int tl = min(t0 + tpc, a.n) - 1, kend = a.pos0 + tl + 1, nstg = (kend + SKEYS - 1) / SKEYS;
    auto load = [&](int buf, int k0) {
        constexpr int KC = DQ / 8, VC = DV / 8;  // 16-byte pieces a row
        const int kc = a.dqk / 8, vc = a.dv / 8;
        for (int i = threadIdx.x; i < SKEYS * (KC + VC); i += NT) {
            const int row = i / (KC + VC), c = i % (KC + VC), key = k0 + row;
            const bool ok = key < kend;
            const int kk = ok ? key : 0;
            if (c < KC)
                cp_async16(ks + (buf * SKEYS + row) * QP + 8 * c,
                           a.k + (size_t)kk * a.ldk + g * a.dqk + 8 * min(c, kc - 1), ok && c < kc);
            else
                cp_async16(vs + (buf * SKEYS + row) * VP + 8 * (c - KC),
                           a.v + (size_t)kk * a.ldv + g * a.dv + 8 * min(c - KC, vc - 1), ok && c - KC < vc);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    float o[NV][4], m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
#pragma unroll
    for (int n = 0; n < NV; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    load(0, 0);
    for (int b = 0; b < nstg; b++) {
        const int buf = b & 1, k0 = b * SKEYS + kh * AP_KB;  // this key group's 32 keys of the stage
        if (b + 1 < nstg) {
            load(buf ^ 1, (b + 1) * SKEYS);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const uint16_t *kb = ks + (buf * SKEYS + kh * AP_KB) * QP, *vb = vs + (buf * SKEYS + kh * AP_KB) * VP;
        // S = Q K^T for the block's 4 key tiles of 8
        float sc[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll
        for (int s = 0; s < KQ; s++) {
            const int fs = QS ? 0 : s;
            if constexpr (QS) {
                ldsm_x4(fqh[0], qh + qrow * QP + 16 * s + qcol);
                ldsm_x4(fql[0], ql + qrow * QP + 16 * s + qcol);
            }
#pragma unroll
            for (int jp = 0; jp < 2; jp++) {
                uint32_t bk[4];
                ldsm_x4(bk, kb + (16 * jp + mr + (mi >> 1) * 8) * QP + 16 * s + (mi & 1) * 8);
                tcmv::mma_f16(sc[2 * jp], fqh[fs][0], fqh[fs][1], fqh[fs][2], fqh[fs][3], bk[0], bk[1]);
                tcmv::mma_f16(sc[2 * jp], fql[fs][0], fql[fs][1], fql[fs][2], fql[fs][3], bk[0], bk[1]);
                tcmv::mma_f16(sc[2 * jp + 1], fqh[fs][0], fqh[fs][1], fqh[fs][2], fqh[fs][3], bk[2], bk[3]);
                tcmv::mma_f16(sc[2 * jp + 1], fql[fs][0], fql[fs][1], fql[fs][2], fql[fs][3], bk[2], bk[3]);
            }
        }
        // scale, causal mask, online softmax per row
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int key = k0 + 8 * j + 2 * tq + (e & 1), h2 = e >> 1;
                float v = sc[j][e] * a.scale;
                if (key > lim[h2]) v = -INFINITY;
                sc[j][e] = v;
                mx[h2] = fmaxf(mx[h2], v);
            }
        float corr[2];
#pragma unroll
        for (int h2 = 0; h2 < 2; h2++) {
            mx[h2] = fmaxf(mx[h2], __shfl_xor_sync(0xffffffffu, mx[h2], 1));
            mx[h2] = fmaxf(mx[h2], __shfl_xor_sync(0xffffffffu, mx[h2], 2));
            const float mn = fmaxf(m[h2], mx[h2]);
            corr[h2] = mn == -INFINITY ? 1.0f : expf(m[h2] - mn);
            m[h2] = mn;
        }
        float rs[2] = {0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int h2 = e >> 1;
                const float p = m[h2] == -INFINITY ? 0.0f : expf(sc[j][e] - m[h2]);
                sc[j][e] = p;
                rs[h2] += p;
            }
#pragma unroll
        for (int h2 = 0; h2 < 2; h2++) {
            rs[h2] += __shfl_xor_sync(0xffffffffu, rs[h2], 1);
            rs[h2] += __shfl_xor_sync(0xffffffffu, rs[h2], 2);
            l[h2] = l[h2] * corr[h2] + rs[h2];
        }
#pragma unroll
        for (int n = 0; n < NV; n++) o[n][0] *= corr[0], o[n][1] *= corr[0], o[n][2] *= corr[1], o[n][3] *= corr[1];
        // O += P V, P as two k-steps of 16 keys
#pragma unroll
        for (int s2 = 0; s2 < 2; s2++) {
            const uint32_t pa0 = pack_h2(sc[2 * s2][0], sc[2 * s2][1]), pa1 = pack_h2(sc[2 * s2][2], sc[2 * s2][3]);
            const uint32_t pa2 = pack_h2(sc[2 * s2 + 1][0], sc[2 * s2 + 1][1]);
            const uint32_t pa3 = pack_h2(sc[2 * s2 + 1][2], sc[2 * s2 + 1][3]);
#pragma unroll
            for (int n = 0; n < NV; n += 2) {
                uint32_t bv[4];
                ldsm_x4_t(bv, vb + (16 * s2 + mr + (mi & 1) * 8) * VP + 8 * n + (mi >> 1) * 8);
                tcmv::mma_f16(o[n], pa0, pa1, pa2, pa3, bv[0], bv[1]);
                tcmv::mma_f16(o[n + 1], pa0, pa1, pa2, pa3, bv[2], bv[3]);
            }
        }
        __syncthreads();  // the buffer is refilled two stages on
    }
    if constexpr (KS == 2) {
        // key group 1 hands its (m, l, o) of every row to group 0 through shared memory (the
        // key / value buffers are free now), which merges the two softmax halves
        float *mo = reinterpret_cast<float *>(ap_smem), *ml = mo + AP_ROWS * DV;
        if (kh == 1) {
#pragma unroll
            for (int h2 = 0; h2 < 2; h2++) {
                const int r = 16 * rw + gq + 8 * h2;
#pragma unroll
                for (int n = 0; n < NV; n++)
                    *reinterpret_cast<float2 *>(mo + r * DV + 8 * n + 2 * tq) = make_float2(o[n][2 * h2], o[n][2 * h2 + 1]);
                if (tq == 0) ml[2 * r] = m[h2], ml[2 * r + 1] = l[h2];
            }
        }
        __syncthreads();
        if (kh == 1) {
            griddep_launch();
            return;
        }
#pragma unroll
        for (int h2 = 0; h2 < 2; h2++) {
            const int r = 16 * rw + gq + 8 * h2;
            const float m1 = ml[2 * r], l1 = ml[2 * r + 1], mm = fmaxf(m[h2], m1);
            const float c0 = m[h2] == -INFINITY ? 0.0f : expf(m[h2] - mm), c1 = m1 == -INFINITY ? 0.0f : expf(m1 - mm);
            l[h2] = l[h2] * c0 + l1 * c1;
#pragma unroll
            for (int n = 0; n < NV; n++) {
                const float2 u = *reinterpret_cast<const float2 *>(mo + r * DV + 8 * n + 2 * tq);
                o[n][2 * h2] = o[n][2 * h2] * c0 + u.x * c1;
                o[n][2 * h2 + 1] = o[n][2 * h2 + 1] * c0 + u.y * c1;
            }
        }
    }
#pragma unroll
    for (int h2 = 0; h2 < 2; h2++) {
        const int r = 16 * rw + gq + 8 * h2, t = t0 + r / G, hh = g * G + r % G;
        if (r >= tpc * G || t >= a.n) continue;
        const float inv = l[h2] > 0.0f ? 1.0f / l[h2] : 0.0f;
        float *dst = a.out + (size_t)t * a.ldo + hh * a.dv + 2 * tq;
#pragma unroll
        for (int n = 0; n < NV; n++)
            if (8 * n < a.dv)
                *reinterpret_cast<float2 *>(dst + 8 * n) = make_float2(o[n][2 * h2] * inv, o[n][2 * h2 + 1] * inv);
    }
    griddep_launch();
}

template <int KQ, int NV, bool QS, int KS = QS ? 1 : 2>
inline int attn_prefill_launch(const AttnPrefillArgs &a, dim3 grid, cudaStream_t s)
{
    constexpr size_t smem = attn_prefill_smem<KQ, NV, QS, KS>();
    static size_t rec[64];
    static std::mutex mu;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (tcmv::ensure_smem(attn_prefill_kernel<KQ, NV, QS, KS>, smem, rec)) return -3;
    }
    return launch_k(attn_prefill_kernel<KQ, NV, QS, KS>, grid, dim3(KS * AP_WARPS * 32), smem, 1, s, a);
}

// The kernel width class of (q width, v width): 0 none, else a case of attn_prefill.
inline int attn_prefill_class(int dqk, int dv)
{
    if (dqk < 8 || dv < 8 || dqk % 8 || dv % 8 || dqk > AP_MAXD || dv > AP_MAXD) return 0;
    if (dqk <= 64 && dv <= 64) return 1;                // (4, 8)
    if (dv <= 128) return dqk <= 96 ? 2 : dqk <= 128 ? 3 : dqk <= 192 ? 4 : 5;  // (6|8|12, 16), (16, 16) QS
    return 6;                                           // (16, 32) QS
}

// Whether attn_prefill takes a (q width, v width, group) shape: widths multiples of 8 up to
// 256 (the reference's block attention takes hd <= 256, group <= 16:
// crates/soso-llm-api/src/cuda.rs:1562-1564), 1 <= group <= 64.
inline bool attn_prefill_takes(int dqk, int dv, int group)
{
    return attn_prefill_class(dqk, dv) != 0 && group >= 1 && group <= AP_ROWS;
}

inline int attn_prefill(const AttnPrefillArgs &a, cudaStream_t s)
{
    if (a.kv_heads < 1 || a.heads % a.kv_heads || !attn_prefill_takes(a.dqk, a.dv, a.heads / a.kv_heads) ||
        a.n < 1 || a.ldk % 8 || a.ldv % 8 || a.ldq % 4 || ((uintptr_t)a.q & 15))
        return -1;
    const int tpc = AP_ROWS / (a.heads / a.kv_heads);
    const dim3 grid((unsigned)((a.n + tpc - 1) / tpc), (unsigned)a.kv_heads);
    switch (attn_prefill_class(a.dqk, a.dv)) {
    case 1: return attn_prefill_launch<4, 8, false>(a, grid, s);    // head_dim 64
    case 2: return attn_prefill_launch<6, 16, false>(a, grid, s);   // MLA: qk 96, v 128
    case 3: return attn_prefill_launch<8, 16, false>(a, grid, s);   // head_dim 128
    case 4: return attn_prefill_launch<12, 16, false>(a, grid, s);  // MLA: qk 192, v 128
    case 5: return attn_prefill_launch<16, 16, true>(a, grid, s);
    case 6: return attn_prefill_launch<16, 32, true>(a, grid, s);   // head_dim 256
    }
    return -5;
}

// ---- MLA -----------------------------------------------------------------------------
// Latent rows of the block: f16 with the reference's rounding (kv.rs:293-315) at pos0 + t.
__global__ void mla_latent_rows_kernel(const float *__restrict__ c, uint16_t *__restrict__ latent, int n, int r,
                                       int pos0)
{
    griddep_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * r; i += gridDim.x * blockDim.x)
        latent[(size_t)(pos0 + i / r) * r + i % r] = f32_to_f16_ref(c[i]);
    griddep_launch();
}

// RoPE (llama pairs, rope_inplace, gemm.rs:1346) of the rope slice of each head of row t at
// position p0 + t: x [rows][heads][qk] f32, slice [qk_nope, qk), freq_i = theta^(-2i/qk_rope).
// With k16 set the whole row goes to f16 (the expanded keys of the attention) and, for
// positions >= krope_from, the roped slice to the rope-key cache krope [ctx][heads][qk_rope].
__global__ void mla_rope_rows_kernel(float *x, int heads, int qk_nope, int qk_rope, int p0, float theta,
                                     uint16_t *k16, float *krope, int krope_from)
{
    griddep_wait();
    const int t = blockIdx.x, qk = qk_nope + qk_rope, pos = p0 + t;
    float *row = x + (size_t)t * heads * qk;
    for (int i = threadIdx.x; i < heads * (qk_rope / 2); i += blockDim.x) {
        const int h = i / (qk_rope / 2), g = i % (qk_rope / 2);
        float *v = row + h * qk + qk_nope + 2 * g;
        const float freq = powf(theta, -2.0f * (float)g / (float)qk_rope);
        const float ang = (float)pos * freq, sn = sinf(ang), cs = cosf(ang);
        const float k0 = v[0], k1 = v[1];
        v[0] = k0 * cs - k1 * sn;
        v[1] = k0 * sn + k1 * cs;
        if (krope && pos >= krope_from) {
            float *d = krope + ((size_t)pos * heads + h) * qk_rope + 2 * g;
            d[0] = v[0], d[1] = v[1];
        }
    }
    if (k16) {
        __syncthreads();
        for (int i = threadIdx.x; i < heads * qk; i += blockDim.x)
            k16[(size_t)t * heads * qk + i] = __half_as_ushort(__float2half_rn(row[i]));
    }
    griddep_launch();
}

// ---- MoE -----------------------------------------------------------------------------
constexpr int MOE_MAXE = 1024, MOE_MAXK = 16;

// Router logits of a block against an f32 matrix (the reference's router matvec,
// layer.rs:1959-1972; mo_router_logits, gemma_capa.cu:517-538): one warp per
// (expert, token), lanes over the hidden size, a fixed-order reduction.
__global__ void router_logits_f32_kernel(const float *__restrict__ w, const float *__restrict__ xs,
                                         float *__restrict__ out, int n_exp, int h)
{
    griddep_wait();
    const int e = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), t = blockIdx.y, lane = threadIdx.x & 31;
    if (e < n_exp) {
        const float *wr = w + (size_t)e * h, *x = xs + (size_t)t * h;
        float acc = 0.0f;
        for (int i = lane; i < h; i += 32) acc += wr[i] * x[i];
        acc = warp_sum(acc);
        if (lane == 0) out[(size_t)t * n_exp + e] = acc;
    }
    griddep_launch();
}

// Grouping of the block's routed pairs p = t * k + j by expert (idx from the router): slot
// order is expert-major, within an expert arbitrary (every row of a GEMM is computed alone,
// so the order changes no value).  Writes pair -> slot, slot -> token, and the two tile
// tables of the expert GEMMs: gate|up pair matrices (rows_gu each, output f16 silu(g)*u per
// slot) and downs (rows_dn each, f32 per slot), tiles of BN tokens, with their counts.
struct GroupArgs {
    const int *idx;  // [n][k]
    int n, k, n_exp, bn;
    int rows_gu, rows_dn;
    int map_gu, map_dn, out_gu, out_dn;  // expert e's maps: map_gu + e, map_dn + e
    int *pair_slot;   // [n k]
    int *slot_tok;    // [n k]
    pg::Tile *t_gu, *t_dn;
    int *n_gu, *n_dn;  // tile counts
    int cap_gu, cap_dn;
};

__global__ void __launch_bounds__(1024) moe_group_kernel(GroupArgs a)
{
    __shared__ int cnt[MOE_MAXE], off[MOE_MAXE], cur[MOE_MAXE], tg[MOE_MAXE], td[MOE_MAXE];
    griddep_wait();
    const int np = a.n * a.k;
    for (int e = threadIdx.x; e < a.n_exp; e += blockDim.x) cnt[e] = 0, cur[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < np; p += blockDim.x) {
        const int e = a.idx[p];
        if (e >= 0 && e < a.n_exp) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int s = 0, sg = 0, sd = 0;
        const int rg = (a.rows_gu + pg::BM - 1) / pg::BM, rd = (a.rows_dn + pg::BM - 1) / pg::BM;
        for (int e = 0; e < a.n_exp; e++) {
            off[e] = s, tg[e] = sg, td[e] = sd;
            const int tt = (cnt[e] + a.bn - 1) / a.bn;
            s += cnt[e], sg += rg * tt, sd += rd * tt;
        }
        *a.n_gu = min(sg, a.cap_gu);
        *a.n_dn = min(sd, a.cap_dn);
        if (sg > a.cap_gu || sd > a.cap_dn) set_dev_error(0x92u);
    }
    __syncthreads();
    for (int p = threadIdx.x; p < np; p += blockDim.x) {
        const int e = a.idx[p];
        if (e < 0 || e >= a.n_exp) {
            a.pair_slot[p] = -1;
            set_dev_error(0x93u);
            continue;
        }
        const int s = off[e] + atomicAdd(&cur[e], 1);
        a.pair_slot[p] = s;
        a.slot_tok[s] = p / a.k;
    }
    // tiles: per expert, row tiles x token tiles, row tile fastest (one token tile's CTAs
    // read the expert's rows in order)
    for (int e = threadIdx.x; e < a.n_exp; e += blockDim.x) {
        const int tt = (cnt[e] + a.bn - 1) / a.bn;
        const int rg = (a.rows_gu + pg::BM - 1) / pg::BM, rd = (a.rows_dn + pg::BM - 1) / pg::BM;
        for (int j = 0; j < tt; j++) {
            const int tok0 = off[e] + j * a.bn, ntok = min(a.bn, cnt[e] - j * a.bn);
            for (int r = 0; r < rg; r++) {
                const int i = tg[e] + j * rg + r;
                if (i < a.cap_gu) a.t_gu[i] = pg::Tile{a.map_gu + e, a.out_gu, r * pg::BM, tok0, ntok, 0, 0, 0};
            }
            for (int r = 0; r < rd; r++) {
                const int i = td[e] + j * rd + r;
                if (i < a.cap_dn) a.t_dn[i] = pg::Tile{a.map_dn + e, a.out_dn, r * pg::BM, tok0, ntok, 0, 0, 0};
            }
        }
    }
    griddep_launch();
}

// Inputs of the routed pairs: row slot = x16 row of its token.
__global__ void moe_gather16_kernel(const __half *__restrict__ x16, const int *__restrict__ slot_tok,
                                    __half *__restrict__ xg, int np, int h)
{
    griddep_wait();
    const int s = blockIdx.x;
    if (s < np) {
        const uint4 *src = reinterpret_cast<const uint4 *>(x16 + (size_t)slot_tok[s] * h);
        uint4 *dst = reinterpret_cast<uint4 *>(xg + (size_t)s * h);
        for (int i = threadIdx.x; i < h / 8; i += blockDim.x) dst[i] = src[i];
    }
    griddep_launch();
}

// The MoE FFN's output added to the residual, per token (forward_moe_ffn, layer.rs:1922-1933,
// :1389): acc = sum over j in choice order of y[slot(t, j)] * w[t][j], then the shared
// expert's output times sigmoid(sg . x) (or 1), h_out = acc + h.
struct CombineArgs {
    const float *h;        // [n][H]
    const float *yd;       // [slots][H]
    const int *pair_slot;  // [n k]
    const float *wts;      // [n][k]
    const float *ysh;      // [n][H] shared expert output, or null
    const float *sg;       // [H] shared gate row, or null (weight 1)
    const float *x32;      // [n][H] the normalised input (for the shared gate)
    float *h_out;          // [n][H]
    int H, k;
};

__global__ void moe_combine_rows_kernel(CombineArgs a)
{
    __shared__ float red[32];
    __shared__ float pgs;
    griddep_wait();
    const int t = blockIdx.x;
    float pg_ = 1.0f;
    if (a.ysh && a.sg) {
        float d = 0.0f;
        for (int i = threadIdx.x; i < a.H; i += blockDim.x) d += a.sg[i] * a.x32[(size_t)t * a.H + i];
        d = warp_sum(d);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = d;
        __syncthreads();
        if (threadIdx.x == 0) {
            float s = 0.0f;
            for (int k = 0; k < (int)(blockDim.x >> 5); k++) s += red[k];
            pgs = 1.0f / (1.0f + expf(-s));
        }
        __syncthreads();
        pg_ = pgs;
    }
    for (int i = threadIdx.x; i < a.H; i += blockDim.x) {
        float acc = 0.0f;
        for (int j = 0; j < a.k; j++) {
            const int s = a.pair_slot[t * a.k + j];
            if (s >= 0) acc += a.yd[(size_t)s * a.H + i] * a.wts[t * a.k + j];
        }
        if (a.ysh) acc += a.ysh[(size_t)t * a.H + i] * pg_;
        a.h_out[(size_t)t * a.H + i] = acc + a.h[(size_t)t * a.H + i];
    }
    griddep_launch();
}

}  // namespace blk
}  // namespace sb
