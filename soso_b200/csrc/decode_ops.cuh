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
// Flash-decoding over the f16 cache, one CTA per (chunk of ATT_CH positions,
// kv head) covering the G = heads/kv_heads query heads that share that kv
// head, so every K/V row is read once per group (like the reference's
// mo_attn_split, gemma_capa.cu:765-877).  Each CTA writes (acc, max, sum) for
// its chunk; the last CTA of a kv head to finish (counter, no spinning) merges
// the chunks in chunk order, as combinar_trozos does (attn_grupo.rs:171-203):
// score = (q.k) / sqrt(hd), softmax over positions 0..pos inclusive.
constexpr int ATT_CH = 64;
constexpr int ATT_THREADS = 256;
constexpr int ATT_MAXG = 8;

struct AttnArgs {
    const float *q;            // [heads][hd], roped
    const uint16_t *kc, *vc;   // [ctx][kv_dim] f16
    float *out;                // [heads][hd]
    float *part;               // workspace [kv_heads][max_chunks][G][hd + 2]
    unsigned *cnt;             // workspace [kv_heads], zero between launches
    const int *pos;
    int heads, kv_heads, kv_dim, ctx, max_chunks;
};

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(AttnArgs a)
{
    __shared__ float qs[ATT_MAXG][HD];
    __shared__ float sc[ATT_MAXG][ATT_CH];
    __shared__ int is_last;
    griddep_wait();
    const int G = a.heads / a.kv_heads, kvh = blockIdx.y, c = blockIdx.x, tid = threadIdx.x;
    const int seq = *a.pos + 1;
    const int nch = (seq + ATT_CH - 1) / ATT_CH;
    if (c >= nch || seq > a.ctx || nch > a.max_chunks) {
        if (c == 0 && tid == 0 && (seq > a.ctx || nch > a.max_chunks)) set_dev_error(0x62u);
        return;
    }
    const int t0 = c * ATT_CH, tn = min(ATT_CH, seq - t0);
    const float inv = 1.0f / sqrtf((float)HD);
    for (int i = tid; i < G * HD; i += ATT_THREADS) qs[i / HD][i % HD] = a.q[(kvh * G) * HD + i];
    __syncthreads();
    // scores: thread (t = tid/4, quarter dq = tid%4)
    {
        const int t = tid >> 2, dq = tid & 3;
        float part[ATT_MAXG];
#pragma unroll
        for (int j = 0; j < ATT_MAXG; j++) part[j] = 0.0f;
        if (t < tn) {
            const uint16_t *krow = a.kc + (size_t)(t0 + t) * a.kv_dim + kvh * HD + dq * (HD / 4);
#pragma unroll
            for (int v8 = 0; v8 < HD / 32; v8++) {
                const uint4 kk = *reinterpret_cast<const uint4 *>(krow + v8 * 8);
                const uint32_t kw[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float2 kf = __half22float2(*reinterpret_cast<const __half2 *>(&kw[e]));
                    const int d = dq * (HD / 4) + v8 * 8 + 2 * e;
#pragma unroll
                    for (int j = 0; j < ATT_MAXG; j++)
                        if (j < G) part[j] += qs[j][d] * kf.x + qs[j][d + 1] * kf.y;
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
    // softmax pieces: warp j owns head j
    const int warp = tid >> 5, lane = tid & 31;
    float *dst = a.part + ((size_t)(kvh * a.max_chunks + c) * G) * (HD + 2);
    if (warp < G) {
        const float s0 = sc[warp][lane], s1 = sc[warp][lane + 32];
        float m = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float p0 = lane < tn ? expf(s0 - m) : 0.0f, p1 = lane + 32 < tn ? expf(s1 - m) : 0.0f;
        sc[warp][lane] = p0;
        sc[warp][lane + 32] = p1;
        const float l = warp_sum(p0 + p1);
        if (lane == 0) {
            dst[warp * (HD + 2) + HD] = m;
            dst[warp * (HD + 2) + HD + 1] = l;
        }
    }
    __syncthreads();
    // P.V: thread -> dims (2*(tid % (HD/2)), +1), heads tid/(HD/2), + step
    {
        const int dp = tid % (HD / 2), j0 = tid / (HD / 2), jstep = ATT_THREADS / (HD / 2);
        for (int j = j0; j < G; j += jstep) {
            float ax = 0.0f, ay = 0.0f;
            for (int t = 0; t < tn; t++) {
                const float p = sc[j][t];
                const float2 vf = __half22float2(
                    *reinterpret_cast<const __half2 *>(a.vc + (size_t)(t0 + t) * a.kv_dim + kvh * HD + 2 * dp));
                ax += p * vf.x;
                ay += p * vf.y;
            }
            dst[j * (HD + 2) + 2 * dp] = ax;
            dst[j * (HD + 2) + 2 * dp + 1] = ay;
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(&a.cnt[kvh], 1u) == (unsigned)(nch - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // merge chunks 0..nch-1 in order (combinar_trozos)
    const float *base = a.part + (size_t)kvh * a.max_chunks * G * (HD + 2);
    for (int i = tid; i < G * HD; i += ATT_THREADS) {
        const int j = i / HD, d = i % HD;
        float mmax = -INFINITY;
        for (int cc = 0; cc < nch; cc++) {
            const float *pc = base + ((size_t)cc * G + j) * (HD + 2);
            if (__ldcg(pc + HD + 1) > 0.0f) mmax = fmaxf(mmax, __ldcg(pc + HD));
        }
        float o = 0.0f, l = 0.0f;
        for (int cc = 0; cc < nch; cc++) {
            const float *pc = base + ((size_t)cc * G + j) * (HD + 2);
            const float li = __ldcg(pc + HD + 1);
            if (li <= 0.0f) continue;
            const float w = expf(__ldcg(pc + HD) - mmax);
            l += w * li;
            o += w * __ldcg(pc + d);
        }
        a.out[(kvh * G + j) * HD + d] = l > 0.0f ? o * (1.0f / l) : 0.0f;
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
// max_by keeps the LAST of equal maxima.  Per-CTA partials, the last CTA to
// finish reduces them (counter, no spinning).
struct ArgmaxArgs {
    const float *v;
    int n;
    float *pv;       // workspace [grid]
    int *pi;         // workspace [grid]
    unsigned *cnt;   // workspace, zero between launches
    int *out;
};

__device__ __forceinline__ void amax_merge(float &bv, int &bi, float v, int i)
{
    if (v > bv || (v == bv && i > bi)) {
        bv = v;
        bi = i;
    }
}

__global__ void argmax_kernel(ArgmaxArgs a)
{
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ int is_last;
    griddep_wait();
    int s, e;
    row_strip(a.n, blockIdx.x, gridDim.x, s, e);
    float bv = -INFINITY;
    int bi = -1;
    for (int i = s + threadIdx.x; i < e; i += blockDim.x) amax_merge(bv, bi, a.v[i], i);
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
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) amax_merge(bv, bi, sv[w], si[w]);
        a.pv[blockIdx.x] = bv;
        a.pi[blockIdx.x] = bi;
        __threadfence();
        is_last = atomicAdd(a.cnt, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (is_last && threadIdx.x == 0) {
        __threadfence();
        float v = -INFINITY;
        int i = -1;
        for (int c = 0; c < (int)gridDim.x; c++) amax_merge(v, i, __ldcg(a.pv + c), __ldcg(a.pi + c));
        *a.out = i < 0 ? 0 : i;
        *a.cnt = 0u;
    }
    griddep_launch();
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
    const size_t chunks = (ctx + sb::ATT_CH - 1) / sb::ATT_CH;
    return 256 + kv_heads * 4 + kv_heads * chunks * G * (head_dim + 2) * 4;
}

extern "C" int sbk_attn_decode(const float *q, const uint16_t *kcache, const uint16_t *vcache, float *out,
                               const int32_t *pos, size_t heads, size_t kv_heads, size_t head_dim, size_t ctx,
                               void *ws, int pdl, void *stream)
{
    if (!q || !kcache || !vcache || !out || !pos || !ws || !kv_heads || heads % kv_heads) return -1;
    const size_t G = heads / kv_heads;
    if (G > sb::ATT_MAXG || head_dim != 128) return -1;
    const int chunks = (int)((ctx + sb::ATT_CH - 1) / sb::ATT_CH);
    // workspace: [counters (zeroed, left zero)] [partials]
    unsigned *cnt = (unsigned *)ws;
    float *part = (float *)((char *)ws + 256 + kv_heads * 4);
    part = (float *)(((uintptr_t)part + 15) & ~(uintptr_t)15);
    sb::AttnArgs a{q, kcache, vcache, out, part, cnt, pos, (int)heads, (int)kv_heads, (int)(kv_heads * head_dim),
                   (int)ctx, chunks};
    return sb::launch_k(sb::attn_decode_kernel<128>, dim3((unsigned)chunks, (unsigned)kv_heads), dim3(sb::ATT_THREADS),
                        0, pdl, (cudaStream_t)stream, a);
}

extern "C" int sbk_router_topk(const float *logits, size_t n_exp, size_t top_k, int32_t *idx, float *wts, int pdl,
                               void *stream)
{
    if (!logits || !idx || !wts || !n_exp || !top_k || top_k > 64 || top_k > n_exp || n_exp > 4096) return -1;
    return sb::launch_k(sb::router_topk_kernel, dim3(1), dim3(256), n_exp * 4, pdl, (cudaStream_t)stream, logits,
                        (int)n_exp, (int)top_k, idx, wts);
}

extern "C" size_t sbk_argmax_ws_bytes(void) { return 256 + 148 * 8 * 2; }

extern "C" int sbk_argmax(const float *v, size_t n, int32_t *out, void *ws, int pdl, void *stream)
{
    if (!v || !n || !out || !ws || n > (1u << 30)) return -1;
    const int grid = 148;
    unsigned *cnt = (unsigned *)ws;
    float *pv = (float *)((char *)ws + 256);
    int *pi = (int *)((char *)ws + 256 + grid * 8);
    sb::ArgmaxArgs a{v, (int)n, pv, pi, cnt, out};
    return sb::launch_k(sb::argmax_kernel, dim3(grid), dim3(256), 0, pdl, (cudaStream_t)stream, a);
}

extern "C" int sbk_embed_row(const void *table, uint8_t dtype, size_t vocab, size_t hidden, const int32_t *token,
                             float *out, int pdl, void *stream)
{
    if (!table || !token || !out || !hidden) return -1;
    if (dtype != 1 && !sbk_row_bytes(dtype, hidden)) return -1;
    return sb::launch_k(sb::embed_kernel, dim3(1), dim3(256), 0, pdl, (cudaStream_t)stream, (const uint8_t *)table,
                        (int)dtype, (int)vocab, (int)hidden, token, out);
}
