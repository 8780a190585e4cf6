// block.cuh -- the steps of a block prefill between the GEMMs (pgemm.cuh): n tokens at
// positions pos0 .. pos0 + n - 1 through one layer, as the reference's forward_layer_block
// (crates/soso-llm-core/src/layer.rs:1433) runs them.
//
//   norm16_rows      h = a (+ res), x = rmsnorm(h) * w (gemm.rs:93-100, add_f32 :265) into
//                    f16 GEMM operands (and f32 when a shared-expert gate needs it)
//   rope_kv_rows     bias, QK-norm, RoPE and the f16 K/V append of every token
//                    (layer.rs:1146-1193, kv.rs:258-275): the decode step's math per row
//   attn_prefill     causal GQA / MHA attention over the f16 rows, f32 throughout
//                    (attention_decode_f16_tiled_scalar, attn.rs:73-140, per query row;
//                    the reference's block kernel is attn_prefill_f16,
//                    lxdde/ports/nouveau/matvec_iq.cu:507-628)
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
// h / (heads / kv_heads): softmax(q.k / sqrt(dqk)) . v with the running maximum and sum of
// the online softmax, in f32 over the f16 rows.  A CTA takes 32 query rows of one kv head
// (32 / G tokens x the G heads of the group) and streams the keys through shared memory
// 32 at a time; each of its 8 warps keeps 4 rows, the lanes splitting the dimensions.
constexpr int AP_ROWS = 32, AP_KB = 32, AP_WARPS = 8, AP_MAXD = 192;

struct AttnPrefillArgs {
    const float *q;      // [n][heads][dqk] (row stride ldq floats)
    const uint16_t *k;   // key rows: key t, kv head g at k + t * ldk + g * dqk  (f16)
    const uint16_t *v;   // value rows: v + t * ldv + g * dv (f16)
    float *out;          // [n][heads][dv] (row stride ldo floats)
    int n, pos0, heads, kv_heads, dqk, dv, ldq, ldk, ldv, ldo;
    float scale;
};

template <int DQ, int DV>  // dims per lane (dqk = 32 DQ, dv = 32 DV)
__global__ void __launch_bounds__(AP_WARPS * 32) attn_prefill_kernel(AttnPrefillArgs a)
{
    __shared__ __align__(16) uint16_t ks[2][AP_KB][32 * DQ + 8];
    __shared__ __align__(16) uint16_t vs[2][AP_KB][32 * DV + 8];
    griddep_wait();
    const int G = a.heads / a.kv_heads, g = blockIdx.y;
    const int tpc = AP_ROWS / G;  // tokens a CTA
    const int t0 = blockIdx.x * tpc;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // this warp's 4 rows: r = 4 warp + j -> token t0 + r / G, head g G + r % G
    float qv[4][DQ], acc[4][DV], m[4], l[4];
    int lim[4];
    bool live[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int r = 4 * warp + j, t = t0 + r / G, hh = g * G + r % G;
        live[j] = t < a.n;
        lim[j] = live[j] ? a.pos0 + t : -1;  // last key this row attends
        m[j] = -INFINITY, l[j] = 0.0f;
#pragma unroll
        for (int d = 0; d < DQ; d++) qv[j][d] = live[j] ? a.q[(size_t)t * a.ldq + hh * a.dqk + lane * DQ + d] : 0.0f;
#pragma unroll
        for (int d = 0; d < DV; d++) acc[j][d] = 0.0f;
    }
    int tl = min(t0 + tpc, a.n) - 1;
    const int kend = a.pos0 + tl + 1;  // keys the CTA needs
    auto load = [&](int buf, int k0) {
        // K rows: DQ*32 f16 = 4 DQ 16-byte pieces a row; V likewise
        const int kp = 4 * DQ, vp = 4 * DV;
        for (int i = threadIdx.x; i < AP_KB * (kp + vp); i += AP_WARPS * 32) {
            const int row = i / (kp + vp), c = i % (kp + vp), key = k0 + row;
            uint4 val = make_uint4(0, 0, 0, 0);
            if (c < kp) {
                if (key < kend) val = *reinterpret_cast<const uint4 *>(a.k + (size_t)key * a.ldk + g * a.dqk + 8 * c);
                *reinterpret_cast<uint4 *>(&ks[buf][row][8 * c]) = val;
            } else {
                const int cv = c - kp;
                if (key < kend) val = *reinterpret_cast<const uint4 *>(a.v + (size_t)key * a.ldv + g * a.dv + 8 * cv);
                *reinterpret_cast<uint4 *>(&vs[buf][row][8 * cv]) = val;
            }
        }
    };
    const int nblk = (kend + AP_KB - 1) / AP_KB;
    load(0, 0);
    __syncthreads();
    for (int b = 0; b < nblk; b++) {
        const int buf = b & 1, k0 = b * AP_KB;
        if (b + 1 < nblk) load(buf ^ 1, k0 + AP_KB);
        for (int kk = 0; kk < AP_KB; kk++) {
            const int key = k0 + kk;
            float kvf[DQ], vvf[DV];
#pragma unroll
            for (int d = 0; d < DQ; d++) kvf[d] = __half2float(__ushort_as_half(ks[buf][kk][lane * DQ + d]));
#pragma unroll
            for (int d = 0; d < DV; d++) vvf[d] = __half2float(__ushort_as_half(vs[buf][kk][lane * DV + d]));
            float s[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float p = 0.0f;
#pragma unroll
                for (int d = 0; d < DQ; d++) p += qv[j][d] * kvf[d];
                s[j] = p;
            }
#pragma unroll
            for (int o = 16; o; o >>= 1)
#pragma unroll
                for (int j = 0; j < 4; j++) s[j] += __shfl_xor_sync(0xffffffffu, s[j], o);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (key > lim[j]) continue;  // causal: uniform over the warp
                const float sc = s[j] * a.scale;
                const float mn = fmaxf(m[j], sc);
                const float corr = expf(m[j] - mn), p = expf(sc - mn);
                l[j] = l[j] * corr + p;
#pragma unroll
                for (int d = 0; d < DV; d++) acc[j][d] = acc[j][d] * corr + p * vvf[d];
                m[j] = mn;
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
        if (!live[j]) continue;
        const int r = 4 * warp + j, t = t0 + r / G, hh = g * G + r % G;
        const float inv = l[j] > 0.0f ? 1.0f / l[j] : 0.0f;
#pragma unroll
        for (int d = 0; d < DV; d++) a.out[(size_t)t * a.ldo + hh * a.dv + lane * DV + d] = acc[j][d] * inv;
    }
    griddep_launch();
}

inline int attn_prefill(const AttnPrefillArgs &a, cudaStream_t s)
{
    if (a.heads % a.kv_heads || AP_ROWS % (a.heads / a.kv_heads) || a.dqk % 32 || a.dv % 32 ||
        a.dqk > AP_MAXD || a.dv > AP_MAXD || a.n < 1)
        return -1;
    const int tpc = AP_ROWS / (a.heads / a.kv_heads);
    const dim3 grid((unsigned)((a.n + tpc - 1) / tpc), (unsigned)a.kv_heads);
    const int DQ = a.dqk / 32, DV = a.dv / 32;
#define AP_CASE(Q, V) \
    if (DQ == Q && DV == V) return launch_k(attn_prefill_kernel<Q, V>, grid, dim3(AP_WARPS * 32), 0, 1, s, a)
    AP_CASE(4, 4);
    AP_CASE(6, 4);
    AP_CASE(2, 2);
    AP_CASE(3, 4);
#undef AP_CASE
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
