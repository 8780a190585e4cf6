// mla.cuh -- multi-head latent attention (MLA) decode in the absorbed form.
//
// The reference (crates/soso-llm-core/src/arch.rs:51-202, attn.rs:306-404) caches one
// f16 latent row c_t = kv_down . x per token (kv.rs:293-315) and, at every step, for
// every cached t and head, re-expands k = k_up . c_t (RoPE on its rope slice at
// position t) and v = v_up . c_t:
//   score_t = (q_h . k_h(t)) / sqrt(qk_nope + qk_rope),  out_h = sum_t softmax_t * v_h(t).
// With k_up's rows of head h split into W_kn (qk_nope rows) and W_kr (qk_rope rows), and
// v_up's into W_v,h, the same numbers are
//   q_h . k_h(t) = (W_kn^T q_nope,h) . c_t  +  q_rope,h . rope_t(W_kr c_t)
//   out_h        = W_v,h . (sum_t softmax_t * c_t)
// so a decode step needs, per head, one absorbed query qt_h = W_kn^T q_nope,h (kv_rank
// values), the rope keys rope_t(W_kr c_t) once per cached token (kept beside the latent
// cache: kv_heads x qk_rope f32 per token), attention over the latent rows, and one
// small matvec W_v,h . cbar_h at the end -- O(seq * (kv_rank + qk_rope)) per head
// instead of O(seq * kv_rank * (qk + v) ) of re-expansion.
//
// q layout: per head qk_nope + qk_rope values (nope first), the stride the reference's
// MLA assumes when qk_nope + qk_rope == hidden/heads (its parity test dims); with
// DeepSeek-V2-Lite dims (128 + 64 != 2048/16) the reference's own stride overlaps heads,
// so the stride here is always qk_nope + qk_rope.  RoPE: llama pairs (2i, 2i+1) over the
// rope slice, freq_i = theta^(-2i/qk_rope) (rope_inplace, gemm.rs:1346, :1493-1509).
#pragma once
#include "decode_ops.cuh"

namespace sb {
namespace mla {

constexpr int THREADS = 256;
constexpr int CH = 16;        // cached positions per sub-chunk of the attention kernel
constexpr int MAXH = 16;      // query heads per layer (attention keeps 16 x 2 accumulators per thread)
constexpr int MAXC = 64;      // spans per step
constexpr int MAXR = 1024;    // kv_rank
constexpr int MAXRP = 128;    // qk_rope

// One Q4_K weight: element e (0..255) of the 144-byte block (dequant.rs:150-248).
__device__ __forceinline__ float q4k_elem(const uint8_t *blk, int e)
{
    const float d = __half2float(*reinterpret_cast<const __half *>(blk));
    const float dmin = __half2float(*reinterpret_cast<const __half *>(blk + 2));
    const uint8_t *sc = blk + 4;
    const int j = e >> 5, l = e & 31, pair = e >> 6;
    unsigned s_, m_;
    if (j < 4) s_ = sc[j] & 63, m_ = sc[j + 4] & 63;
    else s_ = (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4), m_ = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    const uint8_t qb = blk[16 + pair * 32 + l];
    const float q = (float)((j & 1) ? (qb >> 4) : (qb & 15));
    return (d * (float)s_) * q - dmin * (float)m_;
}

struct AbsorbArgs {
    const float *q;        // [heads][qk_per], nope first (q_up output)
    const float *c;        // [kv_rank] (kv_down output)
    const uint8_t *k_up;   // Q4_K [kv_heads * qk_per][kv_rank]
    uint16_t *latent;      // [ctx][kv_rank] f16: the reference's latent cache (kv.rs:293-315)
    float *krope;          // [ctx][kv_heads][qk_rope]
    float *qt;             // [heads][kv_rank]
    float *qr;             // [heads][qk_rope]
    const int *pos;
    int heads, kv_heads, kv_rank, qk_nope, qk_rope, ctx;
    float theta;
};

// CTA h: head h's absorbed query and roped q slice; for h < kv_heads also kv head h's
// rope key at pos; CTA 0 appends the latent row.  The rows of k_up that head h needs are
// staged in shared memory first.
__global__ void __launch_bounds__(THREADS) absorb_kernel(AbsorbArgs a)
{
    extern __shared__ __align__(16) uint8_t sm[];
    griddep_launch();  // the next kernel reads this one's output only after its own wait
    griddep_wait();
    const int h = blockIdx.x, tid = threadIdx.x, qk_per = a.qk_nope + a.qk_rope;
    const int pos = *a.pos;
    if (pos < 0 || pos >= a.ctx) {
        if (h == 0 && tid == 0) set_dev_error(0x81u);
        return;
    }
    const int group = a.heads / a.kv_heads, kvh = h / group;
    const int rb = (a.kv_rank / 256) * 144;  // bytes per k_up row
    uint8_t *rows = sm;                                           // [qk_per][rb]
    float *cf = reinterpret_cast<float *>(sm + (size_t)qk_per * rb);  // [kv_rank]
    float *qs = cf + a.kv_rank;                                   // [qk_per]
    // stage head kvh's rows of k_up (contiguous: qk_per rows)
    const uint4 *src = reinterpret_cast<const uint4 *>(a.k_up + (size_t)kvh * qk_per * rb);
    for (int i = tid; i < qk_per * rb / 16; i += THREADS) reinterpret_cast<uint4 *>(rows)[i] = src[i];
    // the latent row as the cache holds it (f16, the reference's rounding)
    for (int j = tid; j < a.kv_rank; j += THREADS) {
        const uint16_t hb = f32_to_f16_ref(a.c[j]);
        cf[j] = f16_to_f32(hb);
        if (h == 0) a.latent[(size_t)pos * a.kv_rank + j] = hb;
    }
    for (int i = tid; i < qk_per; i += THREADS) qs[i] = a.q[(size_t)h * qk_per + i];
    __syncthreads();
    // roped q slice (pairs 2i, 2i+1)
    for (int i = tid; i < a.qk_rope / 2; i += THREADS) {
        const float freq = powf(a.theta, -2.0f * (float)i / (float)a.qk_rope);
        const float ang = (float)pos * freq, sn = sinf(ang), cs = cosf(ang);
        const float x0 = qs[a.qk_nope + 2 * i], x1 = qs[a.qk_nope + 2 * i + 1];
        a.qr[(size_t)h * a.qk_rope + 2 * i] = x0 * cs - x1 * sn;
        a.qr[(size_t)h * a.qk_rope + 2 * i + 1] = x0 * sn + x1 * cs;
    }
    // absorbed query: qt[j] = sum_i W_kn[i][j] * q_nope[i], i in row order
    for (int j = tid; j < a.kv_rank; j += THREADS) {
        const int b = j >> 8, e = j & 255;
        float acc = 0.0f;
        for (int i = 0; i < a.qk_nope; i++) acc += q4k_elem(rows + (size_t)i * rb + b * 144, e) * qs[i];
        a.qt[(size_t)h * a.kv_rank + j] = acc;
    }
    if (h >= a.kv_heads) return;
    // rope key of kv head h at pos: rows qk_nope.. of its k_up rows times the latent row,
    // one warp per row (lanes over the columns, fixed order), then the rotation
    __shared__ float kr[MAXRP];
    const int warp = tid >> 5, lane = tid & 31;
    for (int i = warp; i < a.qk_rope; i += THREADS / 32) {
        const uint8_t *row = rows + (size_t)(a.qk_nope + i) * rb;
        float acc = 0.0f;
        for (int j = lane; j < a.kv_rank; j += 32) acc += q4k_elem(row + (j >> 8) * 144, j & 255) * cf[j];
        acc = warp_sum(acc);
        if (lane == 0) kr[i] = acc;
    }
    __syncthreads();
    for (int i = tid; i < a.qk_rope / 2; i += THREADS) {
        const float freq = powf(a.theta, -2.0f * (float)i / (float)a.qk_rope);
        const float ang = (float)pos * freq, sn = sinf(ang), cs = cosf(ang);
        const float x0 = kr[2 * i], x1 = kr[2 * i + 1];
        float *dst = a.krope + ((size_t)pos * a.kv_heads + h) * a.qk_rope;
        dst[2 * i] = x0 * cs - x1 * sn;
        dst[2 * i + 1] = x0 * sn + x1 * cs;
    }
}

struct AttnArgs {
    const float *qt;         // [heads][kv_rank]
    const float *qr;         // [heads][qk_rope]
    const uint16_t *latent;  // [ctx][kv_rank] f16
    const float *krope;      // [ctx][kv_heads][qk_rope]
    float *cbar;             // [heads][kv_rank]: sum_t softmax_t * c_t
    float *part;             // workspace [MAXC][heads][kv_rank + 2]
    unsigned *cnt;           // workspace counter, zero between launches
    const int *pos;
    int heads, kv_heads, kv_rank, qk_rope, ctx, span;
    float scale;             // 1 / sqrt(qk_nope + qk_rope)
};

// One CTA per span of cached positions, all heads: the latent rows are read once for every
// head.  Thread (head = tid / CH, t = tid % CH) forms one score per sub-chunk; each head's
// softmax runs online; thread tid accumulates latent dims 2*tid, 2*tid + 1 (and + 512 ..)
// of every head.  Spans are merged like the GQA kernel's (combinar_trozos,
// attn_grupo.rs:171-203).
__global__ void __launch_bounds__(THREADS) attn_kernel(AttnArgs a)
{
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ float s_m[MAXH], s_l[MAXH], s_f[MAXH];
    __shared__ float sc[MAXH][CH];
    __shared__ float sw[MAXH][MAXC];
    __shared__ int is_last;
    // the position was written by the previous token's last kernel (complete before this
    // token's first kernel passed its wait): spans without work leave before waiting
    const int c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pos = __ldcg(a.pos), seq = pos + 1, nch = (seq + a.span - 1) / a.span;
    if (pos < 0 || seq > a.ctx || nch > MAXC || c >= nch) {
        if (c == 0 && tid == 0 && (pos < 0 || seq > a.ctx || nch > MAXC)) set_dev_error(0x82u);
        return;
    }
    griddep_launch();
    griddep_wait();  // the absorbed query and this token's latent row come from the previous kernel
    const int R = a.kv_rank, RP = a.qk_rope, H = a.heads, LS = R + 8;  // padded latent row (halfs)
    float *qt = reinterpret_cast<float *>(sm);                // [H][R]
    float *qr = qt + (size_t)H * R;                           // [H][RP]
    float *kr = qr + (size_t)H * RP;                          // [CH][kv_heads][RP]
    uint16_t *lat = reinterpret_cast<uint16_t *>(kr + (size_t)CH * a.kv_heads * RP);  // [CH][LS]
    for (int i = tid; i < H * R; i += THREADS) qt[i] = a.qt[i];
    for (int i = tid; i < H * RP; i += THREADS) qr[i] = a.qr[i];
    if (tid < MAXH) s_m[tid] = -INFINITY, s_l[tid] = 0.0f;
    const int tb = c * a.span, te = min(seq, tb + a.span);
    const int group = H / a.kv_heads;
    const int NJ = R / (2 * THREADS);  // latent dim pairs per thread (1 or 2)
    float acc[MAXH][2][2];
#pragma unroll
    for (int h = 0; h < MAXH; h++)
#pragma unroll
        for (int k = 0; k < 2; k++) acc[h][k][0] = acc[h][k][1] = 0.0f;
    for (int t0 = tb; t0 < te; t0 += CH) {
        const int tn = min(CH, te - t0);
        __syncthreads();  // previous sub-chunk done with lat / kr / sc
        for (int i = tid; i < tn * (R / 8); i += THREADS) {
            const int r = i / (R / 8), v = i % (R / 8);
            *reinterpret_cast<uint4 *>(lat + (size_t)r * LS + v * 8) =
                *reinterpret_cast<const uint4 *>(a.latent + (size_t)(t0 + r) * R + v * 8);
        }
        for (int i = tid; i < tn * a.kv_heads * RP; i += THREADS) kr[i] = a.krope[(size_t)t0 * a.kv_heads * RP + i];
        __syncthreads();
        {
            const int h = tid / CH, t = tid % CH;
            if (h < H) {
                float s = -INFINITY;
                if (t < tn) {
                    const float *q = qt + (size_t)h * R;
                    const uint16_t *l = lat + (size_t)t * LS;
                    float d = 0.0f;
                    for (int j = 0; j < R; j += 2) {
                        const float2 lf = __half22float2(*reinterpret_cast<const __half2 *>(l + j));
                        d += q[j] * lf.x + q[j + 1] * lf.y;
                    }
                    const float *qrh = qr + (size_t)h * RP, *krh = kr + ((size_t)t * a.kv_heads + h / group) * RP;
                    float dr = 0.0f;
                    for (int j = 0; j < RP; j++) dr += qrh[j] * krh[j];
                    s = (d + dr) * a.scale;
                }
                sc[h][t] = s;
            }
        }
        __syncthreads();
        // online softmax, two heads per warp: lanes 0-15 head 2w, 16-31 head 2w+1
        {
            const int h = 2 * warp + (lane >> 4), t = lane & 15;
            if (h < H) {
                const float s = sc[h][t];
                float m = s;
#pragma unroll
                for (int o = 8; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                const float mo = s_m[h], mn = fmaxf(mo, m);
                const float p = t < tn ? expf(s - mn) : 0.0f;
                float l = p;
#pragma unroll
                for (int o = 8; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
                sc[h][t] = p;
                __syncwarp();
                if (t == 0) {
                    const float f = mo == -INFINITY ? 0.0f : expf(mo - mn);
                    s_f[h] = f;
                    s_l[h] = s_l[h] * f + l;
                    s_m[h] = mn;
                }
            }
        }
        __syncthreads();
        for (int k = 0; k < NJ; k++) {
            const int j = 2 * tid + 2 * THREADS * k;
#pragma unroll
            for (int h = 0; h < MAXH; h++) {
                if (h >= H) break;
                const float f = s_f[h];
                float x0 = acc[h][k][0] * f, y0 = acc[h][k][1] * f;
                for (int t = 0; t < tn; t++) {
                    const float p = sc[h][t];
                    const float2 lf = __half22float2(*reinterpret_cast<const __half2 *>(lat + (size_t)t * LS + j));
                    x0 += p * lf.x;
                    y0 += p * lf.y;
                }
                acc[h][k][0] = x0, acc[h][k][1] = y0;
            }
        }
    }
    __syncthreads();
    if (nch == 1) {
        for (int k = 0; k < NJ; k++) {
            const int j = 2 * tid + 2 * THREADS * k;
#pragma unroll
            for (int h = 0; h < MAXH; h++) {
                if (h >= H) break;
                const float l = s_l[h], r = l > 0.0f ? 1.0f / l : 0.0f;
                a.cbar[(size_t)h * R + j] = acc[h][k][0] * r;
                a.cbar[(size_t)h * R + j + 1] = acc[h][k][1] * r;
            }
        }
        return;
    }
    float *dst = a.part + (size_t)c * H * (R + 2);
    for (int k = 0; k < NJ; k++) {
        const int j = 2 * tid + 2 * THREADS * k;
#pragma unroll
        for (int h = 0; h < MAXH; h++) {
            if (h >= H) break;
            dst[(size_t)h * (R + 2) + j] = acc[h][k][0];
            dst[(size_t)h * (R + 2) + j + 1] = acc[h][k][1];
        }
    }
    if (tid < H) dst[(size_t)tid * (R + 2) + R] = s_m[tid], dst[(size_t)tid * (R + 2) + R + 1] = s_l[tid];
    __threadfence();
    __syncthreads();
    if (tid == 0) is_last = atomicAdd(a.cnt, 1u) == (unsigned)(nch - 1);
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // merge spans: per head weights exp(m_c - M) (one half-warp per head), then the sums
    {
        const int h = 2 * warp + (lane >> 4), t = lane & 15;
        if (h < H) {
            float M = -INFINITY;
            for (int cc = t; cc < nch; cc += 16) {
                const float *pc = a.part + ((size_t)cc * H + h) * (R + 2);
                if (__ldcg(pc + R + 1) > 0.0f) M = fmaxf(M, __ldcg(pc + R));
            }
#pragma unroll
            for (int o = 8; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            float L = 0.0f;
            for (int cc = t; cc < nch; cc += 16) {
                const float *pc = a.part + ((size_t)cc * H + h) * (R + 2);
                const float li = __ldcg(pc + R + 1);
                const float w = li > 0.0f ? expf(__ldcg(pc + R) - M) : 0.0f;
                sw[h][cc] = w;
                L += w * li;
            }
#pragma unroll
            for (int o = 8; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
            if (t == 0) s_l[h] = L;
        }
    }
    __syncthreads();
    for (int i = tid; i < H * R; i += THREADS) {
        const int h = i / R, j = i % R;
        float o = 0.0f;
        for (int cc = 0; cc < nch; cc++) o += sw[h][cc] * __ldcg(a.part + ((size_t)cc * H + h) * (R + 2) + j);
        const float L = s_l[h];
        a.cbar[i] = L > 0.0f ? o * (1.0f / L) : 0.0f;
    }
    if (tid == 0) *a.cnt = 0u;
}

inline size_t absorb_smem(int kv_rank, int qk_per) { return (size_t)qk_per * (kv_rank / 256) * 144 + (kv_rank + qk_per) * 4 + 16; }
inline size_t attn_smem(int heads, int kv_heads, int kv_rank, int qk_rope)
{
    return ((size_t)heads * kv_rank + (size_t)heads * qk_rope + (size_t)CH * kv_heads * qk_rope) * 4 +
           (size_t)CH * (kv_rank + 8) * 2 + 16;
}

}  // namespace mla
}  // namespace sb

extern "C" size_t sbk_mla_ws_bytes(size_t heads, size_t kv_rank)
{
    return 256 + (size_t)sb::mla::MAXC * heads * (kv_rank + 2) * 4;
}

extern "C" int sbk_mla_absorb(const float *q, const float *c, const void *k_up, uint8_t k_up_dtype, uint16_t *latent,
                              float *krope, float *qt, float *qr, const int32_t *pos, size_t heads, size_t kv_heads,
                              size_t kv_rank, size_t qk_nope, size_t qk_rope, size_t ctx, float theta, int pdl,
                              void *stream)
{
    using namespace sb::mla;
    if (!q || !c || !k_up || !latent || !krope || !qt || !qr || !pos) return -1;
    if (k_up_dtype != SB_DTYPE_Q4_K) return -5;
    if (!heads || !kv_heads || heads % kv_heads || heads > MAXH || kv_rank % 256 || kv_rank > MAXR || !qk_nope ||
        !qk_rope || qk_rope % 2 || qk_rope > MAXRP || !ctx)
        return -1;
    if (((uintptr_t)k_up) & 15) return -2;
    const size_t smem = absorb_smem((int)kv_rank, (int)(qk_nope + qk_rope));
    if (smem > 227 * 1024) return -1;
    static size_t rec[64];
    if (sb::tcmv::ensure_smem(absorb_kernel, smem, rec)) return -3;
    AbsorbArgs a{q, c, (const uint8_t *)k_up, latent, krope, qt, qr, pos, (int)heads, (int)kv_heads, (int)kv_rank,
                 (int)qk_nope, (int)qk_rope, (int)ctx, theta};
    return sb::launch_k(absorb_kernel, dim3((unsigned)heads), dim3(THREADS), smem, pdl, (cudaStream_t)stream, a);
}

extern "C" int sbk_mla_attn(const float *qt, const float *qr, const uint16_t *latent, const float *krope, float *cbar,
                            const int32_t *pos, size_t heads, size_t kv_heads, size_t kv_rank, size_t qk_nope,
                            size_t qk_rope, size_t ctx, void *ws, int pdl, void *stream)
{
    using namespace sb::mla;
    if (!qt || !qr || !latent || !krope || !cbar || !pos || !ws) return -1;
    if (!heads || !kv_heads || heads % kv_heads || heads > MAXH || kv_rank % 512 || kv_rank > MAXR || !qk_rope ||
        qk_rope > MAXRP || !ctx || ctx > (1u << 24))
        return -1;
    if (((uintptr_t)latent | (uintptr_t)ws) & 15) return -2;
    const size_t smem = attn_smem((int)heads, (int)kv_heads, (int)kv_rank, (int)qk_rope);
    if (smem > 227 * 1024) return -1;
    static size_t rec[64];
    if (sb::tcmv::ensure_smem(attn_kernel, smem, rec)) return -3;
    const size_t subs = (ctx + CH - 1) / CH;
    const int span = (int)(((subs + MAXC - 1) / MAXC) * CH);
    const int chunks = (int)((ctx + span - 1) / span);
    AttnArgs a{qt, qr, latent, krope, cbar, (float *)((char *)ws + 256), (unsigned *)ws, pos, (int)heads,
               (int)kv_heads, (int)kv_rank, (int)qk_rope, (int)ctx, span, 1.0f / sqrtf((float)(qk_nope + qk_rope))};
    return sb::launch_k(attn_kernel, dim3((unsigned)chunks), dim3(THREADS), smem, pdl, (cudaStream_t)stream, a);
}
