// decode_ops.cuh -- the non-matvec kernels of one decode step on sm_100a:
//   * rope_kv:   q/k/v bias + per-head QK-norm + RoPE + f16 KV append
//   * attention: split-K GQA decode attention over the f16 [token][kv_dim] cache
//   * router:    softmax over all experts, stable top-k, renormalise
//   * argmax:    greedy token (ties -> last index)
//   * embed:     dequantise one embedding row
// All of them read the decode position from device memory, so one captured
// CUDA graph serves every step.
#pragma once
#include "common.cuh"
#include "group.cuh"

namespace sb {

// f32 -> f16 exactly as crates/soso-llm-core/src/f16.rs:10-37 (round to nearest,
// ties away from zero in magnitude, flush below 2^-25), so cached K/V bits match
// the reference's KV cache for the same f32 input.
__device__ __forceinline__ uint16_t f32_to_f16_ref(float v)
{
    const uint32_t bits = __float_as_uint(v);
    const uint32_t sign = (bits >> 16) & 0x8000u;
    const int exp = (int)((bits >> 23) & 0xffu);
    const uint32_t frac = bits & 0x7fffffu;
    if (exp == 255) return (uint16_t)(sign | 0x7c00u | (frac ? 0x200u : 0u));
    const int e = exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        const uint32_t f = frac | 0x800000u, shift = (uint32_t)(14 - e);
        const uint32_t sub = f >> shift, round = (f >> (shift - 1)) & 1u;
        return (uint16_t)(sign | (sub + round));
    }
    const uint32_t half = ((uint32_t)e << 10) | (frac >> 13);
    const uint32_t round = (frac >> 12) & 1u;
    return (uint16_t)((sign | half) + round);
}

__device__ __forceinline__ float f16_to_f32(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// ------------------------------------------------------------------ rope_kv
// One CTA per head: q heads, then k heads, then v heads of the stacked
// [q | k | v] vector.  Order of the reference layer (layer.rs:1146-1193):
// bias (add_optional_bias) -> QK-norm (rmsnorm per head, FLAG_QK_NORM) -> RoPE
// (rope_cabezas, gemm.rs:1452-1491; NeoX pairs (i, i+d/2) or llama pairs
// (2i, 2i+1)) -> append f16 K/V rows at `pos` (kv.rs:258-275).
struct RopeKvArgs {
    float *qkv;
    const float *bias;   // same layout as qkv or null
    const float *qnorm;  // [hd] or null
    const float *knorm;  // [hd] or null
    uint16_t *kc, *vc;   // f16 cache rows [ctx][kv_heads*hd]
    const int *pos;      // device position of this token
    int heads, kv_heads, hd, ctx;
    float theta, eps;
    int neox;
};

__global__ void rope_kv_kernel(RopeKvArgs a)
{
    __shared__ float red[32];
    griddep_wait();
    const int h = blockIdx.x, i = threadIdx.x, half = a.hd >> 1;
    const int kvd = a.kv_heads * a.hd;
    const int pos = *a.pos;
    if (pos < 0 || pos >= a.ctx) {
        if (i == 0 && h == 0) set_dev_error(0x61u);
        return;
    }
    int base, kind;  // kind 0 = q, 1 = k, 2 = v
    if (h < a.heads) kind = 0, base = h * a.hd;
    else if (h < a.heads + a.kv_heads) kind = 1, base = a.heads * a.hd + (h - a.heads) * a.hd;
    else kind = 2, base = a.heads * a.hd + kvd + (h - a.heads - a.kv_heads) * a.hd;
    const int e0 = a.neox ? i : 2 * i, e1 = a.neox ? i + half : 2 * i + 1;
    float v0 = a.qkv[base + e0], v1 = a.qkv[base + e1];
    if (a.bias) {
        v0 += a.bias[base + e0];
        v1 += a.bias[base + e1];
    }
    const float *nw = kind == 0 ? a.qnorm : kind == 1 ? a.knorm : nullptr;
    if (nw) {  // uniform per CTA
        float ss = v0 * v0 + v1 * v1;
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if ((i & 31) == 0) red[i >> 5] = ss;
        __syncthreads();
        float t = 0.0f;
        for (int k = 0; k < (int)((blockDim.x + 31) >> 5); k++) t += red[k];
        const float scale = 1.0f / sqrtf(t / (float)a.hd + a.eps);
        v0 = v0 * scale * nw[e0];
        v1 = v1 * scale * nw[e1];
    }
    if (kind < 2) {
        const float freq = powf(a.theta, (-2.0f * (float)i) / (float)a.hd);
        const float ang = (float)pos * freq;
        const float s = sinf(ang), c = cosf(ang);
        const float r0 = v0 * c - v1 * s, r1 = v0 * s + v1 * c;
        if (kind == 0) {
            a.qkv[base + e0] = r0;
            a.qkv[base + e1] = r1;
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

// ---------------------------------------------------------------- attention
// Flash-decoding over the f16 cache.  One CTA per (span of positions, kv head)
// covers the G = heads/kv_heads query heads that share that kv head, so every
// K/V row is read once per group (like the reference's mo_attn_split,
// gemma_capa.cu:765-877).  A span is ATT_CH positions (more when the context is
// longer than ATT_MAXC * ATT_CH), taken ATT_CH at a time: the sub-chunk's K and V
// rows are copied to shared memory with cp.async first (all in flight at once),
// then scores, an online-softmax update and P.V run out of shared memory.  With
// one span the CTA writes the output directly; otherwise each CTA writes
// (acc, max, sum) and the last CTA of a kv head to finish (counter, no
// spinning) merges the spans in order, as combinar_trozos does
// (attn_grupo.rs:171-203): score = (q.k) / sqrt(hd), softmax over 0..pos.
//
// With `rope` set the kernel also does the step before it (layer.rs:1146-1193,
// as rope_kv_kernel): q heads get bias, QK-norm and RoPE into shared memory,
// and the CTA whose span holds position pos forms this token's K and V rows
// the same way, appends them to the caches (f16, the reference's rounding) and
// uses the rounded rows, exactly as the reference attends over its f16 cache.
constexpr int ATT_CH = 64;
constexpr int ATT_THREADS = 256;
constexpr int ATT_MAXG = 8;
constexpr int ATT_MAXC = 64;  // spans per kv head at most
constexpr int ATT_KPAD = 8;   // f16 pad per cached row in shared memory (272-byte rows)
// q in shared memory: 8 floats of padding after every 32, so the four quarter-dims a warp
// reads at once (32 floats apart) fall in different banks
constexpr int ATT_QS = 160;   // floats per head row (128 + 4 * 8)
__host__ __device__ constexpr int att_qi(int d) { return d + ((d >> 5) << 3); }

struct AttnArgs {
    const float *qkv;          // q [heads][hd]; with rope: then k [kv_heads][hd], v [kv_heads][hd]
    const float *bias;         // rope: same layout as qkv, or null
    const float *qnorm;        // rope: [hd] or null
    const float *knorm;        // rope: [hd] or null
    uint16_t *kc, *vc;         // [ctx][kv_dim] f16
    float *out;                // [heads][hd]
    float *part;               // workspace [kv_heads][ATT_MAXC][G][hd + 2]
    unsigned *cnt;             // workspace [kv_heads], zero between launches
    const int *pos;
    int heads, kv_heads, kv_dim, ctx, span;
    float theta, eps;
    int neox, rope;
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(AttnArgs a)
{
    static_assert(HD == 128, "one lane per two RoPE pairs; one thread per two P.V dims of two heads");
    __shared__ float qs[ATT_MAXG][ATT_QS];
    __shared__ __align__(16) uint16_t ks[ATT_CH][HD + ATT_KPAD];
    __shared__ __align__(16) uint16_t vs[ATT_CH][HD + ATT_KPAD];
    __shared__ __align__(16) uint16_t knew[HD], vnew[HD];
    __shared__ float sc[ATT_MAXG][ATT_CH];
    __shared__ float rc[HD / 2], rs[HD / 2];
    __shared__ float s_m[ATT_MAXG], s_l[ATT_MAXG], s_f[ATT_MAXG];
    __shared__ float sw[ATT_MAXG][ATT_MAXC];
    __shared__ int is_last;
    griddep_wait();
    const int G = a.heads / a.kv_heads, kvh = blockIdx.y, c = blockIdx.x, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int pos = *a.pos, seq = pos + 1;
    const int nch = (seq + a.span - 1) / a.span;
    if (pos < 0 || c >= nch || seq > a.ctx || nch > ATT_MAXC) {
        if (c == 0 && tid == 0 && (pos < 0 || seq > a.ctx || nch > ATT_MAXC)) set_dev_error(0x62u);
        return;
    }
    const int tb = c * a.span, te = min(seq, tb + a.span);
    const bool own_new = a.rope && c == nch - 1;  // this CTA forms and appends row pos
    // first sub-chunk's rows in flight while q (and the new rows) are prepared
    auto load_rows = [&](int t0, int tn) {
        for (int i = tid; i < tn * (HD / 8); i += ATT_THREADS) {
            const int r = i / (HD / 8), v8 = i % (HD / 8);
            if (own_new && t0 + r == pos) continue;
            const size_t g = (size_t)(t0 + r) * a.kv_dim + kvh * HD + v8 * 8;
            cp_async16(&ks[r][v8 * 8], a.kc + g);
            cp_async16(&vs[r][v8 * 8], a.vc + g);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    load_rows(tb, min(ATT_CH, te - tb));
    // RoPE angles (rope_cabezas: freq_i = theta^(-2i/d), angle = pos * freq_i)
    if (a.rope && tid < HD / 2) {
        const float freq = powf(a.theta, (-2.0f * (float)tid) / (float)HD);
        const float ang = (float)pos * freq;
        rs[tid] = sinf(ang);
        rc[tid] = cosf(ang);
    }
    if (tid < ATT_MAXG) s_m[tid] = -INFINITY, s_l[tid] = 0.0f;
    __syncthreads();
    // q heads of the group (and, for own_new, this token's k and v rows): one warp per
    // vector, lane l holds pairs l and l + 32
    const int ntask = G + (own_new ? 2 : 0);
    for (int task = warp; task < ntask; task += ATT_THREADS / 32) {
        const int kind = task < G ? 0 : task - G + 1;  // 0 q, 1 k, 2 v
        const int base = kind == 0 ? (kvh * G + task) * HD : a.heads * HD + (kind == 2 ? a.kv_dim : 0) + kvh * HD;
        float v[4];
        int e[4];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int p = lane + 32 * h;
            e[2 * h] = a.neox ? p : 2 * p;
            e[2 * h + 1] = a.neox ? p + HD / 2 : 2 * p + 1;
        }
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = a.qkv[base + e[k]];
        if (a.rope) {
            if (a.bias) {
#pragma unroll
                for (int k = 0; k < 4; k++) v[k] += a.bias[base + e[k]];
            }
            const float *nw = kind == 0 ? a.qnorm : kind == 1 ? a.knorm : nullptr;
            if (nw) {
                const float ss = warp_sum((v[0] * v[0] + v[1] * v[1]) + (v[2] * v[2] + v[3] * v[3]));
                const float scale = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
                for (int k = 0; k < 4; k++) v[k] = v[k] * scale * nw[e[k]];
            }
            if (kind < 2) {
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const float cs = rc[lane + 32 * h], sn = rs[lane + 32 * h];
                    const float x0 = v[2 * h], x1 = v[2 * h + 1];
                    v[2 * h] = x0 * cs - x1 * sn;
                    v[2 * h + 1] = x0 * sn + x1 * cs;
                }
            }
        }
        if (kind == 0) {
#pragma unroll
            for (int k = 0; k < 4; k++) qs[task][att_qi(e[k])] = v[k];
        } else {
            uint16_t *row = (kind == 1 ? a.kc : a.vc) + (size_t)pos * a.kv_dim + kvh * HD;
            uint16_t *nrow = kind == 1 ? knew : vnew;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint16_t hb = f32_to_f16_ref(v[k]);
                row[e[k]] = hb;
                nrow[e[k]] = hb;
            }
        }
    }
    const float inv = 1.0f / sqrtf((float)HD);
    // P.V ownership: dims 2*dp, 2*dp+1 of heads j0 and j0 + 4
    const int dp = tid % (HD / 2), j0 = tid / (HD / 2);
    float ax[2] = {0.0f, 0.0f}, ay[2] = {0.0f, 0.0f};
    for (int t0 = tb; t0 < te; t0 += ATT_CH) {
        const int tn = min(ATT_CH, te - t0);
        if (t0 != tb) load_rows(t0, tn);
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();  // rows landed; q and the new rows written
        if (own_new && pos >= t0 && pos < t0 + tn)
            for (int i = tid; i < HD; i += ATT_THREADS) ks[pos - t0][i] = knew[i], vs[pos - t0][i] = vnew[i];
        __syncthreads();
        // scores: thread (t = tid/4, quarter dq = tid%4)
        {
            const int t = tid >> 2, dq = tid & 3;
            float part[ATT_MAXG];
#pragma unroll
            for (int j = 0; j < ATT_MAXG; j++) part[j] = 0.0f;
            if (t < tn) {
#pragma unroll
                for (int v8 = 0; v8 < HD / 32; v8++) {
                    const uint4 kk = *reinterpret_cast<const uint4 *>(&ks[t][dq * (HD / 4) + v8 * 8]);
                    const uint32_t kw[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
                    for (int e2 = 0; e2 < 4; e2++) {
                        const float2 kf = __half22float2(*reinterpret_cast<const __half2 *>(&kw[e2]));
                        const int d = att_qi(dq * (HD / 4) + v8 * 8 + 2 * e2);
#pragma unroll
                        for (int j = 0; j < ATT_MAXG; j++)
                            if (j < G) {
                                const float2 qv = *reinterpret_cast<const float2 *>(&qs[j][d]);
                                part[j] += qv.x * kf.x + qv.y * kf.y;
                            }
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < ATT_MAXG; j++) {
                part[j] += __shfl_xor_sync(0xffffffffu, part[j], 1);
                part[j] += __shfl_xor_sync(0xffffffffu, part[j], 2);
            }
            if (dq == 0)
                for (int j = 0; j < G; j++) sc[j][t] = t < tn ? part[j] * inv : -INFINITY;
        }
        __syncthreads();
        // online softmax: warp j owns head j
        if (warp < G) {
            const float s0 = sc[warp][lane], s1 = sc[warp][lane + 32];
            float m = fmaxf(s0, s1);
#pragma unroll
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float mo = s_m[warp], mn = fmaxf(mo, m);
            const float p0 = lane < tn ? expf(s0 - mn) : 0.0f, p1 = lane + 32 < tn ? expf(s1 - mn) : 0.0f;
            sc[warp][lane] = p0;
            sc[warp][lane + 32] = p1;
            const float l = warp_sum(p0 + p1);
            __syncwarp();
            if (lane == 0) {
                const float f = mo == -INFINITY ? 0.0f : expf(mo - mn);
                s_f[warp] = f;
                s_l[warp] = s_l[warp] * f + l;
                s_m[warp] = mn;
            }
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int j = j0 + 4 * h;
            if (j >= G) continue;
            const float f = s_f[j];
            float x0 = ax[h] * f, y0 = ay[h] * f;
            for (int t = 0; t < tn; t++) {
                const float p = sc[j][t];
                const float2 vf = __half22float2(*reinterpret_cast<const __half2 *>(&vs[t][2 * dp]));
                x0 += p * vf.x;
                y0 += p * vf.y;
            }
            ax[h] = x0, ay[h] = y0;
        }
        __syncthreads();  // before the next sub-chunk overwrites ks / vs / sc
    }
    if (nch == 1) {  // the whole context in one span: normalise and store
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int j = j0 + 4 * h;
            if (j >= G) continue;
            const float l = s_l[j], r = l > 0.0f ? 1.0f / l : 0.0f;
            float *o = a.out + (size_t)(kvh * G + j) * HD;
            o[2 * dp] = l > 0.0f ? ax[h] * r : 0.0f;
            o[2 * dp + 1] = l > 0.0f ? ay[h] * r : 0.0f;
        }
        griddep_launch();
        return;
    }
    float *dst = a.part + ((size_t)(kvh * ATT_MAXC + c) * G) * (HD + 2);
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int j = j0 + 4 * h;
        if (j >= G) continue;
        dst[j * (HD + 2) + 2 * dp] = ax[h];
        dst[j * (HD + 2) + 2 * dp + 1] = ay[h];
    }
    if (tid < G) dst[tid * (HD + 2) + HD] = s_m[tid], dst[tid * (HD + 2) + HD + 1] = s_l[tid];
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(&a.cnt[kvh], 1u) == (unsigned)(nch - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // merge spans 0..nch-1 (combinar_trozos): per head, weights exp(m_c - M) from one warp,
    // then every output element as an independent-load sum over spans
    const float *base = a.part + (size_t)kvh * ATT_MAXC * G * (HD + 2);
    // (m, l) of every span read once (two spans per lane at most: ATT_MAXC = 64)
    if (warp < G) {
        const int j = warp;
        float mv[2], lv[2];
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int cc = lane + 32 * u;
            const float *pc = base + ((size_t)cc * G + j) * (HD + 2);
            lv[u] = cc < nch ? __ldcg(pc + HD + 1) : 0.0f;
            mv[u] = cc < nch ? __ldcg(pc + HD) : -INFINITY;
        }
        float M = fmaxf(lv[0] > 0.0f ? mv[0] : -INFINITY, lv[1] > 0.0f ? mv[1] : -INFINITY);
#pragma unroll
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float L = 0.0f;
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int cc = lane + 32 * u;
            const float w = lv[u] > 0.0f ? expf(mv[u] - M) : 0.0f;
            if (cc < nch) sw[j][cc] = w;
            L += w * lv[u];
        }
        L = warp_sum(L);
        if (lane == 0) s_l[j] = L;
    }
    __syncthreads();
    // every thread sums its G*HD/ATT_THREADS outputs together, span by span, so the loads of
    // one span (and of the next few) are all in flight at once
    constexpr int PER = ATT_MAXG * HD / ATT_THREADS;  // 4
    float o[PER];
#pragma unroll
    for (int u = 0; u < PER; u++) o[u] = 0.0f;
#pragma unroll 4
    for (int cc = 0; cc < nch; cc++) {
#pragma unroll
        for (int u = 0; u < PER; u++) {
            const int i = tid + u * ATT_THREADS, j = i / HD, d = i % HD;
            if (j < G) o[u] += sw[j][cc] * __ldcg(base + ((size_t)cc * G + j) * (HD + 2) + d);
        }
    }
#pragma unroll
    for (int u = 0; u < PER; u++) {
        const int i = tid + u * ATT_THREADS, j = i / HD, d = i % HD;
        if (j < G) {
            const float L = s_l[j];
            a.out[(kvh * G + j) * HD + d] = L > 0.0f ? o[u] * (1.0f / L) : 0.0f;
        }
    }
    if (tid == 0) a.cnt[kvh] = 0u;
    griddep_launch();
}

// ------------------------------------------------------------------- router
// gemm::topk_softmax (crates/soso-llm-core/src/gemm.rs:62-91): softmax over all
// experts, stable sort by weight descending (ties keep the lower index first),
// keep k, renormalise by their sum (in rank order).  One CTA.
__global__ void router_topk_kernel(const float *__restrict__ logits, int n, int k, int *__restrict__ idx,
                                   float *__restrict__ wts)
{
    extern __shared__ float p[];
    __shared__ float red[32];
    griddep_wait();
    const int tid = threadIdx.x;
    float m = -INFINITY;
    for (int i = tid; i < n; i += blockDim.x) m = fmaxf(m, logits[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    m = -INFINITY;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) m = fmaxf(m, red[w]);
    __syncthreads();
    float s = 0.0f;
    for (int i = tid; i < n; i += blockDim.x) {
        p[i] = expf(logits[i] - m);
        s += p[i];
    }
    s = warp_sum(s);
    if ((tid & 31) == 0) red[tid >> 5] = s;
    __syncthreads();
    s = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[w];
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x)
        if (s > 0.0f) p[i] = p[i] / s;
    __syncthreads();
    __shared__ float topw[64];
    for (int i = tid; i < n; i += blockDim.x) {
        const float v = p[i];
        int r = 0;
        for (int j = 0; j < n; j++) {
            const float u = p[j];
            r += (u > v) || (u == v && j < i);
        }
        if (r < k) {
            idx[r] = i;
            topw[r] = v;
        }
    }
    __syncthreads();
    if (tid == 0) {
        float t = 0.0f;
        for (int r = 0; r < k; r++) t += topw[r];
        for (int r = 0; r < k; r++) wts[r] = t > 0.0f ? topw[r] / t : topw[r];
    }
    griddep_launch();
}

// ------------------------------------------------------------------- argmax
// Runtime::argmax (crates/soso-llm-core/src/runtime.rs:2021-2028): Rust's
// max_by keeps the LAST of equal maxima.  Per-CTA partials (four independent
// loads in flight per thread), the last CTA to finish reduces them in parallel
// (counter, no spinning).  When `step` is set it also ends a greedy step of the
// device-side loop: hist[i] = the argmax of step i, the next token is prompt[i+1]
// while the prompt lasts, else that argmax; the position advances.
constexpr int AM_THREADS = 512;
constexpr int AM_GRID = 148;

struct ArgmaxArgs {
    const float *v;
    int n;
    float *pv;       // workspace [grid]
    int *pi;         // workspace [grid]
    unsigned *cnt;   // workspace, zero between launches
    int *out;
    // greedy step (all null when unused)
    int *pos, *step, *hist;
    const int *prompt, *n_prompt;
    // tensor-parallel: v is this rank's vocabulary slice starting at `base`; the slice's
    // (max, index) goes to every rank's exchange area (pub.dst[p] -> 2 x u32) and
    // argmax_gather_kernel finishes the step
    int base;
    grp::Pub pub;
};

__device__ __forceinline__ void amax_merge(float &bv, int &bi, float v, int i)
{
    if (v > bv || (v == bv && i > bi)) {
        bv = v;
        bi = i;
    }
}

__device__ __forceinline__ void amax_block(float &bv, int &bi, float *sv, int *si)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        amax_merge(bv, bi, ov, oi);
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int nw = blockDim.x >> 5;
        bv = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
        bi = threadIdx.x < nw ? si[threadIdx.x] : -1;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            amax_merge(bv, bi, ov, oi);
        }
    }
}

__global__ void __launch_bounds__(AM_THREADS) argmax_kernel(ArgmaxArgs a)
{
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ int is_last;
    griddep_wait();
    int s, e;
    row_strip(a.n, blockIdx.x, gridDim.x, s, e);
    float bv = -INFINITY;
    int bi = -1;
    for (int i = s + threadIdx.x; i < e; i += 4 * AM_THREADS) {
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = i + k * AM_THREADS < e ? a.v[i + k * AM_THREADS] : -INFINITY;
#pragma unroll
        for (int k = 0; k < 4; k++)
            if (i + k * AM_THREADS < e) amax_merge(bv, bi, v[k], i + k * AM_THREADS);
    }
    amax_block(bv, bi, sv, si);
    if (threadIdx.x == 0) {
        a.pv[blockIdx.x] = bv;
        a.pi[blockIdx.x] = bi;
        __threadfence();
        is_last = atomicAdd(a.cnt, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    bv = -INFINITY, bi = -1;
    for (int c = threadIdx.x; c < (int)gridDim.x; c += AM_THREADS) amax_merge(bv, bi, __ldcg(a.pv + c), __ldcg(a.pi + c));
    __syncthreads();
    amax_block(bv, bi, sv, si);
    if (threadIdx.x == 0 && a.pub.n) {
        const unsigned vb = __float_as_uint(bv), ib = (unsigned)(a.base + (bi < 0 ? 0 : bi));
        for (int p = 0; p < a.pub.n; p++) {
            unsigned *d = reinterpret_cast<unsigned *>(a.pub.dst[p]);
            d[0] = vb;
            d[1] = ib;
        }
        __threadfence_system();
        for (int p = 0; p < a.pub.n; p++) atomicAdd_system(a.pub.cnt[p], 1u);
        *a.cnt = 0u;
    } else if (threadIdx.x == 0) {
        const int tok = bi < 0 ? 0 : bi;
        *a.out = tok;
        *a.cnt = 0u;
        if (a.step) {
            const int i = *a.step;
            a.hist[i] = tok;
            if (i + 1 < *a.n_prompt) *a.out = a.prompt[i + 1];
            *a.pos += 1;
            *a.step = i + 1;
        }
    }
    griddep_launch();
}

// End of a tensor-parallel greedy step: wait for every rank's (max, index) of its vocabulary
// slice, take the largest (ties to the larger index, as Runtime::argmax), record it and feed
// the next token as argmax_kernel does, then start the next epoch.  One thread.
struct GatherArgs {
    void *area;              // own exchange area
    const unsigned *cnt;     // counters of the argmax exchange point, [n]
    unsigned *epoch;
    int n;
    int *out, *pos, *step, *hist;
    const int *prompt, *n_prompt;
};

__global__ void argmax_gather_kernel(GatherArgs a)
{
    griddep_wait();
    if (threadIdx.x != 0) return;
    const unsigned e = *a.epoch;
    grp::wait_counts(a.cnt, a.n, e);
    float bv = -INFINITY;
    int bi = -1;
    for (int s = 0; s < a.n; s++) {
        const unsigned *sl = grp::arg_slot(a.area, s);
        amax_merge(bv, bi, __uint_as_float(__ldcg(sl)), (int)__ldcg(sl + 1));
    }
    const int tok = bi < 0 ? 0 : bi;
    const int i = *a.step;
    a.hist[i] = tok;
    *a.out = i + 1 < *a.n_prompt ? a.prompt[i + 1] : tok;
    *a.pos += 1;
    *a.step = i + 1;
    *a.epoch = e + 1;
}

// -------------------------------------------------------------------- embed
// Runtime::embed_token (runtime.rs:787-802): one row of the embedding table,
// dequantised exactly (dequant.rs decoders).  Token id from device memory.
__global__ void embed_kernel(const uint8_t *__restrict__ table, int dtype, int vocab, int h, const int *tok,
                             float *__restrict__ out)
{
    griddep_wait();
    const int t = *tok;
    if (t < 0 || t >= vocab) {
        if (threadIdx.x == 0) set_dev_error(0x63u);
        return;
    }
    for (int e = threadIdx.x; e < h; e += blockDim.x) {
        float v = 0.0f;
        if (dtype == 1) {
            v = reinterpret_cast<const float *>(table)[(size_t)t * h + e];
        } else if (dtype == 2) {
            const uint8_t *blk = table + ((size_t)t * (h / 32) + e / 32) * 36;
            v = (float)(int8_t)blk[4 + (e & 31)] * __uint_as_float(ldg_u32(blk));
        } else if (dtype == 3) {
            const uint8_t *blk = table + ((size_t)t * (h / 256) + e / 256) * 144;
            const int j = (e & 255) >> 5, l = e & 31, pair = j >> 1;
            const uint8_t *sc = blk + 4;
            unsigned s_, m_;
            if (j < 4) s_ = sc[j] & 63, m_ = sc[j + 4] & 63;
            else s_ = (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4), m_ = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
            const float d = f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            const float dmin = f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
            const uint8_t q = blk[16 + pair * 32 + l];
            v = (d * (float)s_) * (float)((j & 1) ? (q >> 4) : (q & 15)) - dmin * (float)m_;
        } else if (dtype == 13) {
            const uint8_t *blk = table + ((size_t)t * (h / 256) + e / 256) * 210;
            const int r = e & 255, n = r >> 7, rr = r & 127, quarter = rr >> 5, l = rr & 31;
            const uint8_t *ql = blk + n * 64, *qh = blk + 128 + n * 32;
            const int8_t *scp = reinterpret_cast<const int8_t *>(blk + 192 + n * 8);
            const float d = f16_to_f32((uint16_t)(blk[208] | (blk[209] << 8)));
            const int lo = (quarter & 1) ? ql[l + 32] : ql[l];
            const int nib = (quarter >> 1) ? (lo >> 4) : (lo & 15);
            const int q = (nib | (((qh[l] >> (2 * quarter)) & 3) << 4)) - 32;
            v = d * (float)scp[l / 16 + 2 * quarter] * (float)q;
        }
        out[e] = v;
    }
    griddep_launch();
}

}  // namespace sb

// ----------------------------------------------------------- C ABI launchers
namespace sb {
inline cudaLaunchAttribute pdl_attr()
{
    cudaLaunchAttribute a;
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
    return a;
}

template <typename... KArgs, typename... Args>
inline int launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, int pdl, cudaStream_t s, Args... args)
{
    cudaLaunchConfig_t c = {};
    c.gridDim = grid;
    c.blockDim = block;
    c.dynamicSmemBytes = smem;
    c.stream = s;
    cudaLaunchAttribute a[1] = {pdl_attr()};
    c.attrs = a;
    c.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&c, k, args...) == cudaSuccess ? 0 : -4;
}
}  // namespace sb

extern "C" int sbk_rope_kv_append(float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                  uint16_t *kcache, uint16_t *vcache, const int32_t *pos, size_t heads,
                                  size_t kv_heads, size_t head_dim, size_t ctx, float theta, float eps, int neox,
                                  int pdl, void *stream)
{
    if (!qkv || !kcache || !vcache || !pos || !heads || !kv_heads) return -1;
    if (head_dim < 64 || head_dim > 512 || (head_dim / 2) % 32 || heads % kv_heads) return -1;
    sb::RopeKvArgs a{qkv, bias, qnorm, knorm, kcache, vcache, pos, (int)heads, (int)kv_heads, (int)head_dim,
                     (int)ctx, theta, eps, neox};
    return sb::launch_k(sb::rope_kv_kernel, dim3((unsigned)(heads + 2 * kv_heads)), dim3((unsigned)head_dim / 2), 0,
                        pdl, (cudaStream_t)stream, a);
}

extern "C" size_t sbk_attn_ws_bytes(size_t heads, size_t kv_heads, size_t head_dim, size_t ctx)
{
    const size_t G = kv_heads ? heads / kv_heads : 0;
    (void)ctx;
    return 256 + kv_heads * 4 + 16 + kv_heads * sb::ATT_MAXC * G * (head_dim + 2) * 4;
}

namespace sb {
inline int attn_launch(const AttnArgs &a0, size_t heads, size_t kv_heads, size_t head_dim, size_t ctx, void *ws,
                       int pdl, cudaStream_t s)
{
    if (!a0.qkv || !a0.kc || !a0.vc || !a0.out || !a0.pos || !ws || !kv_heads || heads % kv_heads) return -1;
    const size_t G = heads / kv_heads;
    if (G > ATT_MAXG || head_dim != 128 || ctx == 0 || ctx > (1u << 24)) return -1;
    if (((uintptr_t)a0.kc | (uintptr_t)a0.vc) & 15) return -2;
    // positions per CTA: ATT_CH, or a multiple of it so at most ATT_MAXC spans cover ctx
    const size_t subs = (ctx + ATT_CH - 1) / ATT_CH;
    const int span = (int)(((subs + ATT_MAXC - 1) / ATT_MAXC) * ATT_CH);
    const int chunks = (int)((ctx + span - 1) / span);
    // workspace: [counters (zeroed, left zero)] [partials]
    AttnArgs a = a0;
    a.cnt = (unsigned *)ws;
    float *part = (float *)((char *)ws + 256 + kv_heads * 4);
    a.part = (float *)(((uintptr_t)part + 15) & ~(uintptr_t)15);
    a.heads = (int)heads, a.kv_heads = (int)kv_heads, a.kv_dim = (int)(kv_heads * head_dim);
    a.ctx = (int)ctx, a.span = span;
    return launch_k(attn_decode_kernel<128>, dim3((unsigned)chunks, (unsigned)kv_heads), dim3(ATT_THREADS), 0, pdl,
                    s, a);
}
}  // namespace sb

extern "C" int sbk_attn_decode(const float *q, const uint16_t *kcache, const uint16_t *vcache, float *out,
                               const int32_t *pos, size_t heads, size_t kv_heads, size_t head_dim, size_t ctx,
                               void *ws, int pdl, void *stream)
{
    sb::AttnArgs a = {};
    a.qkv = q, a.kc = const_cast<uint16_t *>(kcache), a.vc = const_cast<uint16_t *>(vcache), a.out = out, a.pos = pos;
    a.rope = 0;
    return sb::attn_launch(a, heads, kv_heads, head_dim, ctx, ws, pdl, (cudaStream_t)stream);
}

extern "C" int sbk_attn_rope_decode(const float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                    uint16_t *kcache, uint16_t *vcache, float *out, const int32_t *pos, size_t heads,
                                    size_t kv_heads, size_t head_dim, size_t ctx, float theta, float eps, int neox,
                                    void *ws, int pdl, void *stream)
{
    sb::AttnArgs a = {};
    a.qkv = qkv, a.bias = bias, a.qnorm = qnorm, a.knorm = knorm, a.kc = kcache, a.vc = vcache, a.out = out;
    a.pos = pos, a.theta = theta, a.eps = eps, a.neox = neox, a.rope = 1;
    return sb::attn_launch(a, heads, kv_heads, head_dim, ctx, ws, pdl, (cudaStream_t)stream);
}

extern "C" int sbk_router_topk(const float *logits, size_t n_exp, size_t top_k, int32_t *idx, float *wts, int pdl,
                               void *stream)
{
    if (!logits || !idx || !wts || !n_exp || !top_k || top_k > 64 || top_k > n_exp || n_exp > 4096) return -1;
    return sb::launch_k(sb::router_topk_kernel, dim3(1), dim3(256), n_exp * 4, pdl, (cudaStream_t)stream, logits,
                        (int)n_exp, (int)top_k, idx, wts);
}

extern "C" size_t sbk_argmax_ws_bytes(void) { return 256 + sb::AM_GRID * 8 * 2; }

namespace sb {
inline int argmax_launch(const float *v, size_t n, int32_t *out, void *ws, int pdl, cudaStream_t s, int *pos,
                         int *step, int *hist, const int *prompt, const int *n_prompt)
{
    if (!v || !n || !out || !ws || n > (1u << 30)) return -1;
    unsigned *cnt = (unsigned *)ws;
    float *pv = (float *)((char *)ws + 256);
    int *pi = (int *)((char *)ws + 256 + AM_GRID * 8);
    ArgmaxArgs a{v, (int)n, pv, pi, cnt, out, pos, step, hist, prompt, n_prompt, 0, grp::Pub{}};
    return launch_k(argmax_kernel, dim3(AM_GRID), dim3(AM_THREADS), 0, pdl, s, a);
}
}  // namespace sb

extern "C" int sbk_argmax(const float *v, size_t n, int32_t *out, void *ws, int pdl, void *stream)
{
    return sb::argmax_launch(v, n, out, ws, pdl, (cudaStream_t)stream, nullptr, nullptr, nullptr, nullptr, nullptr);
}

extern "C" int sbk_embed_row(const void *table, uint8_t dtype, size_t vocab, size_t hidden, const int32_t *token,
                             float *out, int pdl, void *stream)
{
    if (!table || !token || !out || !hidden) return -1;
    if (dtype != 1 && !sbk_row_bytes(dtype, hidden)) return -1;
    return sb::launch_k(sb::embed_kernel, dim3(1), dim3(256), 0, pdl, (cudaStream_t)stream, (const uint8_t *)table,
                        (int)dtype, (int)vocab, (int)hidden, token, out);
}
