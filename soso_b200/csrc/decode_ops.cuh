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
#include "tc_mmv.cuh"

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
    const float *factors;  // [hd / 2] divisors of the pair frequencies (YaRN) or null
    float mscale;          // multiplies cos and sin (1: plain RoPE)
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
        float freq = powf(a.theta, (-2.0f * (float)i) / (float)a.hd);
        if (a.factors) freq /= a.factors[i];  // YaRN: the reference's gm_rope (gemma_capa.cu:99-125)
        const float ang = (float)pos * freq;
        const float s = sinf(ang) * a.mscale, c = cosf(ang) * a.mscale;  // mscale 1: exact
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
// Flash-decoding over the f16 cache.  The CTAs of one kv head form a thread-block
// cluster of ATT_SPANS; CTA c takes span c of the positions 0..pos (spans of a
// multiple of ATT_MIN positions, as many as the context needs up to ATT_SPANS) for
// the G = heads/kv_heads query heads that share the kv head, so every K/V row is
// read once per group (like the reference's mo_attn_split, gemma_capa.cu:765-877).
// A span is taken ATT_CH positions at a time through two shared-memory buffers: the
// rows of the next sub-chunk arrive by TMA (2-D tiles of the cache, 64 rows x 64 dims,
// 128-byte swizzle; completion counted on an mbarrier) while the current one is
// computed.  Per sub-chunk, scores
// S = K.q and the output update O += V^T.P run on the tensor cores (mma.sync
// m16n8k16, f32 accumulation) with q and P each split into two f16 parts (hi + lo,
// 22 significant bits; K and V are f16 already), around an online softmax per head
// in f32.  The spans are merged as combinar_trozos does (attn_grupo.rs:171-203) --
// weights exp(m_c - M), sum of l_c, in span order -- by the cluster itself: every
// CTA stores each CTA's share of its partial output into that CTA's shared memory,
// and after one cluster barrier each CTA forms its share of the outputs locally.
//
// With `rope` set the kernel also does the step before it (layer.rs:1146-1193,
// as rope_kv_kernel): q heads get bias, QK-norm and RoPE, and the CTA whose span
// holds position pos forms this token's K and V rows the same way, appends them to
// the caches (f16, the reference's rounding) and uses the rounded rows, exactly as
// the reference attends over its f16 cache.
//
// Everything that does not depend on the previous kernel happens before
// griddepcontrol.wait: the position (written before this kernel's stream position
// by another kernel than the previous one: in the decode graph, the previous
// token's last kernel), the cached rows of earlier positions (the tile holding row
// pos is loaded too; that row is replaced in shared memory by the one this kernel
// forms), the RoPE angles, biases and norm weights.
constexpr int ATT_CH = 64;       // positions per sub-chunk (one K/V buffer)
constexpr int ATT_THREADS = 256;
constexpr int ATT_MAXG = 8;
constexpr int ATT_SPANS = 16;    // CTAs per kv head: one cluster
constexpr int ATT_MIN = 16;      // positions per span at least
constexpr int ATT_HD = 128;
constexpr int ATT_RS = ATT_HD + 8;  // f16 per K/V/q row in shared memory (272 B: ldmatrix rows conflict-free)
constexpr int ATT_PS = ATT_CH + 8;  // f16 per P row (144 B)

// Positions per span for a context of seq positions.
__host__ __device__ inline int att_span(int seq)
{
    const int per = (seq + ATT_SPANS - 1) / ATT_SPANS;
    const int span = (per + ATT_MIN - 1) / ATT_MIN * ATT_MIN;
    return span > ATT_MIN ? span : ATT_MIN;
}

struct AttnArgs {
    CUtensorMap kmap, vmap;    // the caches as [ctx][kv_dim] u16, box ATT_CH rows x 64 dims, 128-byte swizzle
    const float *qkv;          // q [heads][hd]; with rope: then k [kv_heads][hd], v [kv_heads][hd]
    const float *bias;         // rope: same layout as qkv, or null
    const float *qnorm;        // rope: [hd] or null
    const float *knorm;        // rope: [hd] or null
    uint16_t *kc, *vc;         // [ctx][kv_dim] f16
    float *out;                // [heads][hd]
    const int *pos;
    int heads, kv_heads, kv_dim, ctx;
    float theta, eps;
    int neox, rope;
    const float *factors;      // rope: [hd / 2] YaRN divisors of the pair frequencies, or null
    float mscale;              // rope with factors: multiplies cos and sin
};

struct AttSmem {
    uint8_t kb[2][2][ATT_CH * 128];  // [buffer][dims 0-63 | 64-127]: 64 rows x 128 B, 128-byte swizzle
    uint8_t vb[2][2][ATT_CH * 128];
    uint16_t qh[ATT_MAXG][ATT_RS], ql[ATT_MAXG][ATT_RS];  // q = qh + ql (f16 parts)
    uint16_t ph[ATT_MAXG][ATT_PS], pl[ATT_MAXG][ATT_PS];  // P = ph + pl
    float sc[ATT_MAXG][ATT_CH];
    // merge: this CTA's share of the outputs (ATT_MAXG * ATT_HD / ATT_SPANS at most) as each
    // span left it, and every span's (max, sum) per head
    float racc[ATT_SPANS][ATT_MAXG * ATT_HD / ATT_SPANS];
    float rm[ATT_SPANS][ATT_MAXG], rl[ATT_SPANS][ATT_MAXG];
    float m[ATT_MAXG], l[ATT_MAXG], f[ATT_MAXG];
    uint16_t knew[ATT_HD], vnew[ATT_HD];
    float rc[ATT_HD / 2], rs[ATT_HD / 2];
    uint64_t bar[2];
};

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t att_swz(int row, int chunk) { return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4)); }

// Address of dims d0..d0+7 (d0 a multiple of 8) of tile row `row` in a [2 halves][8 KB] buffer.
__device__ __forceinline__ const uint8_t *att_at(const uint8_t (*buf)[ATT_CH * 128], int row, int d0)
{
    return buf[d0 >> 6] + att_swz(row, (d0 & 63) >> 3);
}

__device__ __forceinline__ void tma_tile_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(tcmv::smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(tcmv::smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(tcmv::smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(tcmv::smem_u32(p)));
}

// Store v at `p` (this CTA's address of a shared variable) in CTA `rank` of the cluster.
__device__ __forceinline__ void cluster_st_f32(const void *p, int rank, float v)
{
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(tcmv::smem_u32(p)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}

__device__ __forceinline__ void cluster_arrive_relaxed()
{
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait()
{
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// f32 -> f16 hi part and the f16 rounding of the rest
__device__ __forceinline__ void split_f16(float x, uint16_t &hi, uint16_t &lo)
{
    const __half h = __float2half_rn(x);
    hi = __half_as_ushort(h);
    lo = __half_as_ushort(__float2half_rn(x - __half2float(h)));
}

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS, 1) attn_decode_kernel(const __grid_constant__ AttnArgs a)
{
    static_assert(HD == ATT_HD, "one lane per two RoPE pairs; 8 warps x 16 output dims");
    extern __shared__ __align__(1024) uint8_t att_raw[];
    // the swizzled tiles want 1024-byte-aligned addresses (the launch adds 1024 bytes of slack)
    AttSmem &s = *reinterpret_cast<AttSmem *>(att_raw + ((1024u - (tcmv::smem_u32(att_raw) & 1023u)) & 1023u));
    const int G = a.heads / a.kv_heads, kvh = blockIdx.y, c = blockIdx.x, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
    const int pos = __ldcg(a.pos), seq = pos + 1;
    if (pos < 0 || seq > a.ctx) {  // the same for every CTA: all leave
        if (c == 0 && kvh == 0 && tid == 0) set_dev_error(0x62u);
        return;
    }
    const int span = att_span(seq), nch = (seq + span - 1) / span;
    const bool active = c < nch;
    const int tb = c * span, te = active ? min(seq, tb + span) : tb;
    const int nsub = active ? (te - tb + ATT_CH - 1) / ATT_CH : 0;
    const bool own_new = a.rope && c == nch - 1;  // this CTA forms and appends row pos
    if (nch == 1 && !active) return;              // no merge to take part in
    // the next kernel may be scheduled now; it reads the output only after its own wait
    griddep_launch();
    // (a CTA's shared memory may be written by the others only once every CTA of the
    // cluster is running: the first phase of the cluster barrier, waited for before the merge)
    if (nch > 1) cluster_arrive_relaxed();
    if (tid == 0) {
        tcmv::mbar_init(&s.bar[0], 1);
        tcmv::mbar_init(&s.bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // q and P rows of absent heads stay zero; no head has a running max yet
    for (int i = tid; i < (ATT_MAXG - G) * ATT_RS; i += ATT_THREADS)
        (&s.qh[G][0])[i] = 0, (&s.ql[G][0])[i] = 0;
    for (int i = tid; i < (ATT_MAXG - G) * ATT_PS; i += ATT_THREADS) (&s.ph[G][0])[i] = 0, (&s.pl[G][0])[i] = 0;
    if (tid < ATT_MAXG) s.m[tid] = -INFINITY, s.l[tid] = 0.0f, s.f[tid] = 0.0f;
    __syncthreads();
    // rows t0..t0+63 of sub-chunk i into buffer i & 1 (thread 0): four 64 x 64 tiles (rows
    // past ctx read as zero; rows past the sub-chunk are not used)
    auto issue = [&](int i) {
        const int t0 = tb + i * ATT_CH, b = i & 1;
        tcmv::mbar_expect_tx_arrive(&s.bar[b], 4u * ATT_CH * 128);
        for (int h = 0; h < 2; h++) {
            tma_tile_2d(s.kb[b][h], &a.kmap, kvh * HD + 64 * h, t0, &s.bar[b]);
            tma_tile_2d(s.vb[b][h], &a.vmap, kvh * HD + 64 * h, t0, &s.bar[b]);
        }
    };
    if (tid == 0) {
        if (nsub > 0) issue(0);
        if (nsub > 1) issue(1);
    }
    int issued = nsub < 2 ? nsub : 2;
    // RoPE angles (rope_cabezas: freq_i = theta^(-2i/d), angle = pos * freq_i)
    if (active && a.rope && tid < HD / 2) {
        float freq = powf(a.theta, (-2.0f * (float)tid) / (float)HD);
        if (a.factors) freq /= a.factors[tid];  // YaRN as gm_rope takes it (gemma_capa.cu:99-125)
        const float ang = (float)pos * freq;
        s.rs[tid] = a.factors ? sinf(ang) * a.mscale : sinf(ang);
        s.rc[tid] = a.factors ? cosf(ang) * a.mscale : cosf(ang);
    }
    // q heads of the group (and, for own_new, this token's k and v rows): one warp per
    // vector, lane l holds pairs l and l + 32; a warp has two vectors at most
    const int ntask = active ? G + (own_new ? 2 : 0) : 0;
    int e[4];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int p = lane + 32 * h;
        e[2 * h] = a.neox ? p : 2 * p;
        e[2 * h + 1] = a.neox ? p + HD / 2 : 2 * p + 1;
    }
    float cb[2][4], cn[2][4];  // bias and norm weight of each of this warp's vectors
#pragma unroll
    for (int tt = 0; tt < 2; tt++) {
        const int task = warp + tt * (ATT_THREADS / 32);
        const int kind = task < G ? 0 : task - G + 1;  // 0 q, 1 k, 2 v
        const int base = kind == 0 ? (kvh * G + task) * HD : a.heads * HD + (kind == 2 ? a.kv_dim : 0) + kvh * HD;
        const float *nw = kind == 0 ? a.qnorm : kind == 1 ? a.knorm : nullptr;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            cb[tt][k] = task < ntask && a.rope && a.bias ? a.bias[base + e[k]] : 0.0f;
            cn[tt][k] = task < ntask && a.rope && nw ? nw[e[k]] : 1.0f;
        }
    }
    griddep_wait();  // q|k|v are written by the previous kernel
    __syncthreads();
#pragma unroll
    for (int tt = 0; tt < 2; tt++) {
        const int task = warp + tt * (ATT_THREADS / 32);
        if (task >= ntask) break;
        const int kind = task < G ? 0 : task - G + 1;
        const int base = kind == 0 ? (kvh * G + task) * HD : a.heads * HD + (kind == 2 ? a.kv_dim : 0) + kvh * HD;
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] = a.qkv[base + e[k]];
        if (a.rope) {
#pragma unroll
            for (int k = 0; k < 4; k++) v[k] += cb[tt][k];
            const bool normed = kind == 0 ? a.qnorm != nullptr : kind == 1 ? a.knorm != nullptr : false;
            if (normed) {
                const float ss = warp_sum((v[0] * v[0] + v[1] * v[1]) + (v[2] * v[2] + v[3] * v[3]));
                const float scale = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
                for (int k = 0; k < 4; k++) v[k] = v[k] * scale * cn[tt][k];
            }
            if (kind < 2) {
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const float cs = s.rc[lane + 32 * h], sn = s.rs[lane + 32 * h];
                    const float x0 = v[2 * h], x1 = v[2 * h + 1];
                    v[2 * h] = x0 * cs - x1 * sn;
                    v[2 * h + 1] = x0 * sn + x1 * cs;
                }
            }
        }
        if (kind == 0) {
#pragma unroll
            for (int k = 0; k < 4; k++) split_f16(v[k], s.qh[task][e[k]], s.ql[task][e[k]]);
        } else {
            uint16_t *row = (kind == 1 ? a.kc : a.vc) + (size_t)pos * a.kv_dim + kvh * HD;
            uint16_t *nrow = kind == 1 ? s.knew : s.vnew;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint16_t hb = f32_to_f16_ref(v[k]);
                row[e[k]] = hb;
                nrow[e[k]] = hb;
            }
        }
    }
    __syncthreads();
    const float inv = 1.0f / sqrtf((float)HD);
    // O^T accumulator of warp w: dims 16w + g8 (+ 8) x heads 2*t4, 2*t4 + 1
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int mi = lane >> 3, mr = lane & 7;  // ldmatrix: matrix and row this lane addresses
    bool failed = false;
    int done = 0;
    for (int i = 0; i < nsub; i++) {
        const int t0 = tb + i * ATT_CH, tn = min(ATT_CH, te - t0), b = i & 1;
        if (!tcmv::mbar_wait(&s.bar[b], (unsigned)(i >> 1) & 1u)) failed = true;
        if (__syncthreads_or(failed)) {
            failed = true;
            break;
        }
        done = i + 1;
        if (own_new && pos >= t0 && pos < t0 + tn && tid < HD) {  // this token's rows
            const int r = pos - t0, d = tid;
            const uint32_t o = att_swz(r, (d & 63) >> 3) + (d & 7) * 2;
            *reinterpret_cast<uint16_t *>(s.kb[b][d >> 6] + o) = s.knew[d];
            *reinterpret_cast<uint16_t *>(s.vb[b][d >> 6] + o) = s.vnew[d];
        }
        // rows past the sub-chunk: zero V (P is zero there; other rows could hold non-finite values)
        for (int idx = tid; idx < (ATT_CH - tn) * 64; idx += ATT_THREADS) {
            const int r = tn + idx / 64, w = idx % 64;
            reinterpret_cast<uint32_t *>(s.vb[b][w >> 5] + r * 128)[w & 31] = 0u;
        }
        __syncthreads();
        // scores: warp w < 4 takes positions 16w..16w+15 (rows of the MMA), heads as columns
        if (warp < 4) {
            const int p0 = warp * 16;
            float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (p0 < tn) {
#pragma unroll
                for (int k0 = 0; k0 < HD; k0 += 16) {
                    uint32_t af[4];
                    ldsm_x4(af, att_at(s.kb[b], p0 + (mi & 1) * 8 + mr, k0 + (mi >> 1) * 8));
                    const uint32_t bh0 = *reinterpret_cast<const uint32_t *>(&s.qh[g8][k0 + 2 * t4]);
                    const uint32_t bh1 = *reinterpret_cast<const uint32_t *>(&s.qh[g8][k0 + 2 * t4 + 8]);
                    const uint32_t bl0 = *reinterpret_cast<const uint32_t *>(&s.ql[g8][k0 + 2 * t4]);
                    const uint32_t bl1 = *reinterpret_cast<const uint32_t *>(&s.ql[g8][k0 + 2 * t4 + 8]);
                    tcmv::mma_f16(d, af[0], af[1], af[2], af[3], bh0, bh1);
                    tcmv::mma_f16(d, af[0], af[1], af[2], af[3], bl0, bl1);
                }
            }
            const int pa = p0 + g8, pb = pa + 8, h0 = 2 * t4, h1 = h0 + 1;
            if (h0 < G) {
                s.sc[h0][pa] = pa < tn ? d[0] * inv : -INFINITY;
                s.sc[h0][pb] = pb < tn ? d[2] * inv : -INFINITY;
            }
            if (h1 < G) {
                s.sc[h1][pa] = pa < tn ? d[1] * inv : -INFINITY;
                s.sc[h1][pb] = pb < tn ? d[3] * inv : -INFINITY;
            }
        }
        __syncthreads();
        // online softmax: warp j owns head j; P as f16 parts
        if (warp < G) {
            const float s0 = s.sc[warp][lane], s1 = s.sc[warp][lane + 32];
            float m = fmaxf(s0, s1);
#pragma unroll
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float mo = s.m[warp], mn = fmaxf(mo, m);
            const float p0 = lane < tn ? expf(s0 - mn) : 0.0f, p1 = lane + 32 < tn ? expf(s1 - mn) : 0.0f;
            split_f16(p0, s.ph[warp][lane], s.pl[warp][lane]);
            split_f16(p1, s.ph[warp][lane + 32], s.pl[warp][lane + 32]);
            const float l = warp_sum(p0 + p1);
            if (lane == 0) {
                const float f = mo == -INFINITY ? 0.0f : expf(mo - mn);
                s.f[warp] = f;
                s.l[warp] = s.l[warp] * f + l;
                s.m[warp] = mn;
            }
        }
        __syncthreads();
        // O^T (dims x heads) = f * O^T + V^T . P^T: warp w takes dims 16w..16w+15
        {
            const float fa = s.f[2 * t4], fb = s.f[2 * t4 + 1];
            acc[0] *= fa, acc[1] *= fb, acc[2] *= fa, acc[3] *= fb;
            const int d0 = warp * 16;
            for (int k0 = 0; k0 < tn; k0 += 16) {
                uint32_t af[4];
                ldsm_x4_t(af, att_at(s.vb[b], k0 + (mi >> 1) * 8 + mr, d0 + (mi & 1) * 8));
                const uint32_t bh0 = *reinterpret_cast<const uint32_t *>(&s.ph[g8][k0 + 2 * t4]);
                const uint32_t bh1 = *reinterpret_cast<const uint32_t *>(&s.ph[g8][k0 + 2 * t4 + 8]);
                const uint32_t bl0 = *reinterpret_cast<const uint32_t *>(&s.pl[g8][k0 + 2 * t4]);
                const uint32_t bl1 = *reinterpret_cast<const uint32_t *>(&s.pl[g8][k0 + 2 * t4 + 8]);
                tcmv::mma_f16(acc, af[0], af[1], af[2], af[3], bh0, bh1);
                tcmv::mma_f16(acc, af[0], af[1], af[2], af[3], bl0, bl1);
            }
        }
        __syncthreads();  // buffer b, the scores and P are free again
        if (tid == 0 && i + 2 < nsub) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(i + 2);
        }
        if (i + 2 < nsub) issued = i + 3;
    }
    if (failed) {
        // let the copies issued into this CTA's shared memory land before leaving (bounded)
        if (tid == 0) {
            set_dev_error(0x64u);
            for (int i = done; i < issued; i++) tcmv::mbar_wait(&s.bar[i & 1], (unsigned)(i >> 1) & 1u);
        }
        __syncthreads();
    }
    {
        const int d0 = warp * 16 + g8, h0 = 2 * t4;
        if (nch == 1) {  // the whole context in one span: normalise and store
            if (h0 < G) {
                const float l = s.l[h0], r = l > 0.0f ? 1.0f / l : 0.0f;
                a.out[(size_t)(kvh * G + h0) * HD + d0] = l > 0.0f ? acc[0] * r : 0.0f;
                a.out[(size_t)(kvh * G + h0) * HD + d0 + 8] = l > 0.0f ? acc[2] * r : 0.0f;
            }
            if (h0 + 1 < G) {
                const float l = s.l[h0 + 1], r = l > 0.0f ? 1.0f / l : 0.0f;
                a.out[(size_t)(kvh * G + h0 + 1) * HD + d0] = l > 0.0f ? acc[1] * r : 0.0f;
                a.out[(size_t)(kvh * G + h0 + 1) * HD + d0 + 8] = l > 0.0f ? acc[3] * r : 0.0f;
            }
            return;
        }
    }
    // merge the spans (combinar_trozos): CTA r of the cluster forms outputs r*per .. r*per+per-1
    // (o = head * HD + dim); every active span stores its share of each CTA's outputs and
    // its (max, sum) per head there, then after one cluster barrier each CTA merges locally
    const int per = G * HD / ATT_SPANS;
    cluster_wait();
    if (active) {
        const int d0 = warp * 16 + g8, h0 = 2 * t4;
        const float v4[4] = {acc[0], acc[1], acc[2], acc[3]};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int h = h0 + (k & 1), d = d0 + 8 * (k >> 1);
            if (h >= G) continue;
            const int o = h * HD + d;
            cluster_st_f32(&s.racc[c][o % per], o / per, v4[k]);
        }
        if (tid < ATT_SPANS * G) {
            const int r = tid / G, j = tid % G;
            cluster_st_f32(&s.rm[c][j], r, s.m[j]);
            cluster_st_f32(&s.rl[c][j], r, s.l[j]);
        }
    }
    cluster_sync();
    if (tid < per) {
        const int o = c * per + tid, j = o / HD, d = o % HD;
        float M = -INFINITY;
        for (int cc = 0; cc < nch; cc++)
            if (s.rl[cc][j] > 0.0f) M = fmaxf(M, s.rm[cc][j]);
        float L = 0.0f, O = 0.0f;
        for (int cc = 0; cc < nch; cc++) {
            const float lv = s.rl[cc][j], w = lv > 0.0f ? expf(s.rm[cc][j] - M) : 0.0f;
            L += w * lv;
            O += w * s.racc[cc][tid];
        }
        a.out[(size_t)(kvh * G + j) * HD + d] = L > 0.0f ? O * (1.0f / L) : 0.0f;
    }
}

// ------------------------------------------------------------------- router
// gemm::topk_softmax (crates/soso-llm-core/src/gemm.rs:62-91): softmax over all
// experts, stable sort by weight descending (ties keep the lower index first),
// keep k, renormalise by their sum (in rank order).  One CTA per token: CTA b routes
// logits row b into idx / wts row b.
__global__ void router_topk_kernel(const float *__restrict__ logits, int n, int k, int *__restrict__ idx,
                                   float *__restrict__ wts)
{
    extern __shared__ float p[];
    __shared__ float red[32];
    griddep_wait();
    logits += (size_t)blockIdx.x * n;
    idx += (size_t)blockIdx.x * k;
    wts += (size_t)blockIdx.x * k;
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
// dequantised exactly (dequant.rs decoders).  Token id from device memory; CTA b
// makes row b of out from tok[b] (one CTA: one token).
__global__ void embed_kernel(const uint8_t *__restrict__ table, int dtype, int vocab, int h, const int *tok,
                             float *__restrict__ out)
{
    griddep_launch();  // the next kernel reads the row only after its own wait
    griddep_wait();
    const int t = tok[blockIdx.x];
    out += (size_t)blockIdx.x * h;
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

extern "C" int sbk_rope_kv_append_yarn(float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                       uint16_t *kcache, uint16_t *vcache, const int32_t *pos, size_t heads,
                                       size_t kv_heads, size_t head_dim, size_t ctx, float theta, float eps, int neox,
                                       const float *factors, float mscale, int pdl, void *stream);

extern "C" int sbk_rope_kv_append(float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                  uint16_t *kcache, uint16_t *vcache, const int32_t *pos, size_t heads,
                                  size_t kv_heads, size_t head_dim, size_t ctx, float theta, float eps, int neox,
                                  int pdl, void *stream)
{
    return sbk_rope_kv_append_yarn(qkv, bias, qnorm, knorm, kcache, vcache, pos, heads, kv_heads, head_dim, ctx,
                                   theta, eps, neox, nullptr, 1.0f, pdl, stream);
}

extern "C" int sbk_rope_kv_append_yarn(float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                       uint16_t *kcache, uint16_t *vcache, const int32_t *pos, size_t heads,
                                       size_t kv_heads, size_t head_dim, size_t ctx, float theta, float eps, int neox,
                                       const float *factors, float mscale, int pdl, void *stream)
{
    if (!qkv || !kcache || !vcache || !pos || !heads || !kv_heads) return -1;
    if (head_dim < 64 || head_dim > 512 || (head_dim / 2) % 32 || heads % kv_heads) return -1;
    if (!(mscale > 0.0f) || !isfinite(mscale)) return -1;
    sb::RopeKvArgs a{qkv,          bias,         qnorm,       knorm, kcache, vcache, pos,     (int)heads,
                     (int)kv_heads, (int)head_dim, (int)ctx,    theta, eps,    neox,   factors, mscale};
    return sb::launch_k(sb::rope_kv_kernel, dim3((unsigned)(heads + 2 * kv_heads)), dim3((unsigned)head_dim / 2), 0,
                        pdl, (cudaStream_t)stream, a);
}

extern "C" size_t sbk_attn_ws_bytes(size_t heads, size_t kv_heads, size_t head_dim, size_t ctx)
{
    // the spans are merged inside each kv head's cluster: no workspace is used (kept for the
    // interface: a caller may pass any buffer)
    (void)heads, (void)kv_heads, (void)head_dim, (void)ctx;
    return 256;
}

namespace sb {
// The cache of one layer as a 2-D tensor for the attention kernel's TMA tiles.
inline int attn_map(CUtensorMap *m, const uint16_t *cache, size_t kv_dim, size_t ctx)
{
    tcmv::EncodeTiledFn fn = tcmv::encode_fn();
    if (!fn) return -6;
    cuuint64_t dims[2] = {(cuuint64_t)kv_dim, (cuuint64_t)ctx};
    cuuint64_t strides[1] = {(cuuint64_t)kv_dim * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)ATT_CH};
    cuuint32_t es[2] = {1, 1};
    const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t *>(cache), dims, strides, box, es,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -7;
}

inline int attn_launch(const AttnArgs &a0, size_t heads, size_t kv_heads, size_t head_dim, size_t ctx, void *ws,
                       int pdl, cudaStream_t s)
{
    (void)ws;
    if (!a0.qkv || !a0.kc || !a0.vc || !a0.out || !a0.pos || !kv_heads || heads % kv_heads) return -1;
    const size_t G = heads / kv_heads;
    if (G > ATT_MAXG || head_dim != ATT_HD || ctx == 0 || ctx > (1u << 24) || kv_heads > 65535) return -1;
    if (((uintptr_t)a0.kc | (uintptr_t)a0.vc) & 15) return -2;
    // one cluster of ATT_SPANS CTAs per kv head (a non-portable cluster size)
    static size_t smem_rec[64];
    static std::mutex mu;
    {
        std::lock_guard<std::mutex> lk(mu);
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64) return -3;
        if (!smem_rec[dev]) {
            if (cudaFuncSetAttribute(attn_decode_kernel<ATT_HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)sizeof(AttSmem) + 1024) != cudaSuccess ||
                cudaFuncSetAttribute(attn_decode_kernel<ATT_HD>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
                    cudaSuccess)
                return -3;
            smem_rec[dev] = sizeof(AttSmem);
        }
    }
    AttnArgs a = a0;
    a.heads = (int)heads, a.kv_heads = (int)kv_heads, a.kv_dim = (int)(kv_heads * head_dim);
    a.ctx = (int)ctx;
    int rc = attn_map(&a.kmap, a.kc, kv_heads * head_dim, ctx);
    if (!rc) rc = attn_map(&a.vmap, a.vc, kv_heads * head_dim, ctx);
    if (rc) return rc;
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((unsigned)ATT_SPANS, (unsigned)kv_heads);
    c.blockDim = dim3(ATT_THREADS);
    c.dynamicSmemBytes = sizeof(AttSmem) + 1024;
    c.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = ATT_SPANS, at[0].val.clusterDim.y = 1, at[0].val.clusterDim.z = 1;
    at[1] = pdl_attr();
    c.attrs = at;
    c.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&c, attn_decode_kernel<ATT_HD>, a) == cudaSuccess ? 0 : -4;
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

extern "C" int sbk_attn_rope_decode_yarn(const float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                         uint16_t *kcache, uint16_t *vcache, float *out, const int32_t *pos,
                                         size_t heads, size_t kv_heads, size_t head_dim, size_t ctx, float theta,
                                         float eps, int neox, const float *factors, float mscale, void *ws, int pdl,
                                         void *stream);

extern "C" int sbk_attn_rope_decode(const float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                    uint16_t *kcache, uint16_t *vcache, float *out, const int32_t *pos, size_t heads,
                                    size_t kv_heads, size_t head_dim, size_t ctx, float theta, float eps, int neox,
                                    void *ws, int pdl, void *stream)
{
    return sbk_attn_rope_decode_yarn(qkv, bias, qnorm, knorm, kcache, vcache, out, pos, heads, kv_heads, head_dim,
                                     ctx, theta, eps, neox, nullptr, 1.0f, ws, pdl, stream);
}

extern "C" int sbk_attn_rope_decode_yarn(const float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                         uint16_t *kcache, uint16_t *vcache, float *out, const int32_t *pos,
                                         size_t heads, size_t kv_heads, size_t head_dim, size_t ctx, float theta,
                                         float eps, int neox, const float *factors, float mscale, void *ws, int pdl,
                                         void *stream)
{
    if (!(mscale > 0.0f) || !isfinite(mscale)) return -1;
    sb::AttnArgs a = {};
    a.qkv = qkv, a.bias = bias, a.qnorm = qnorm, a.knorm = knorm, a.kc = kcache, a.vc = vcache, a.out = out;
    a.pos = pos, a.theta = theta, a.eps = eps, a.neox = neox, a.rope = 1;
    a.factors = factors, a.mscale = mscale;
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
