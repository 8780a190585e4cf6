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

constexpr int AB_THREADS = 512;
constexpr int AB_WARPS = AB_THREADS / 32;
constexpr int AB_RG = AB_THREADS / 8;  // row groups (8 threads a row)
constexpr int AB_ROWS = 4;             // qk_nope rows per thread: qk_nope <= AB_RG * AB_ROWS

// d * scale and dmin * min of sub-block j (0-7) of a Q4_K block whose first 16 bytes are
// `hd` (d, dmin, 12 scale bytes): the 6-bit scale / min unpacking of get_scale_min_k4
// (dequant.rs:150-248: w = (d * sc) * q - dmin * m).
__device__ __forceinline__ void q4k_sub(const uint4 &hd, int j, float &ds, float &dm)
{
    const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xffffu)));
    const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
    const int sh = 8 * (j & 3);
    const unsigned by = (hd.y >> sh) & 255u, bz = (hd.z >> sh) & 255u, bw = (hd.w >> sh) & 255u;
    unsigned s_, m_;
    if (j < 4) s_ = by & 63u, m_ = bz & 63u;
    else s_ = (bw & 15u) | ((by >> 6) << 4), m_ = (bw >> 4) | ((bz >> 6) << 4);
    ds = d * (float)s_;
    dm = dmin * (float)m_;
}

// Grid (kv_rank / 64, heads): CTA (p, h) forms qt_h over latent columns 64p .. 64p + 63 --
// the two sub-blocks (2 * pair, 2 * pair + 1) of Q4_K block p / 4 whose weights share the
// 32 code bytes pair * 32 .. (low / high nibble) -- for every nope row, and for h < kv_heads
// the rope keys of kv head h's rope rows RPC * p .. RPC * p + RPC - 1 (RPC even, so each
// rotated pair stays in one CTA).  CTAs (p, 0) append latent columns 64p .. ; CTA (0, h)
// ropes head h's q slice.  The k_up codes do not depend on the previous kernel: every
// thread loads its share into registers before the dependency wait.
//
// qt: thread (row r0 = tid / 8, code word w4 = tid % 8) holds rows r0, r0 + 64, .. and
// code bytes 4 w4 .. 4 w4 + 3 (8 weights per row); its sums run over its rows in order,
// then over the 4 row groups of a warp (shuffle tree) and the 16 warps (in warp order).
// Rope row i of the CTA: warps i % 8 and i % 8 + 8 take the two halves of its code bytes.
__global__ void __launch_bounds__(AB_THREADS) absorb_kernel(AbsorbArgs a)
{
    __shared__ float red[AB_WARPS][64];
    __shared__ float krp[2][MAXRP];
    __shared__ float cs[MAXR];         // the latent row as the cache holds it (f16 values)
    __shared__ float qs[AB_RG * AB_ROWS];  // q_nope of head h
    griddep_launch();  // the next kernel reads this one's output only after its own wait
    const int p = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qk_per = a.qk_nope + a.qk_rope, kvh = h / (a.heads / a.kv_heads);
    const int nbk = a.kv_rank / 256, rb = nbk * 144, np = nbk * 4;
    const int b = p >> 2, pair = p & 3;
    const uint8_t *W = a.k_up + (size_t)kvh * qk_per * rb;
    const int w4 = tid & 7, r0 = tid >> 3;
    uint4 hd[AB_ROWS];
    uint32_t cw[AB_ROWS];
#pragma unroll
    for (int k = 0; k < AB_ROWS; k++) {
        const int r = r0 + AB_RG * k;
        if (r < a.qk_nope) {
            const uint8_t *blk = W + (size_t)r * rb + b * 144;
            hd[k] = __ldg(reinterpret_cast<const uint4 *>(blk));
            cw[k] = __ldg(reinterpret_cast<const uint32_t *>(blk + 16 + pair * 32 + 4 * w4));
        }
    }
    // rope rows: warp w takes rows w % 8, w % 8 + 8, .. of the CTA, code-byte half w / 8
    // (lane chunk t8 = lane + 32 * half: 8 code bytes 8 (t8 % 16) .. of block t8 / 16)
    const int rpc = ((a.qk_rope + np - 1) / np + 1) & ~1, rlo = rpc * p, rhi = min(a.qk_rope, rlo + rpc);
    const bool rope = h < a.kv_heads && rlo < rhi;
    const uint8_t *WR = a.k_up + (size_t)h * qk_per * rb;  // kv head h's rows (rope keys)
    const int rw0 = warp & 7, t8 = lane + 32 * (warp >> 3);
    const bool rlane = t8 < nbk * 16;
    uint4 rh = make_uint4(0u, 0u, 0u, 0u);
    uint2 rc = make_uint2(0u, 0u);
    if (rope && rw0 < rhi - rlo && rlane) {
        const uint8_t *blk = WR + (size_t)(a.qk_nope + rlo + rw0) * rb + (t8 >> 4) * 144;
        rh = __ldg(reinterpret_cast<const uint4 *>(blk));
        rc = __ldg(reinterpret_cast<const uint2 *>(blk + 16 + 8 * (t8 & 15)));
    }
    griddep_wait();  // q (q_up) and c (kv_down) come from the previous kernels
    // one round of loads: pos, the latent row, q_nope and (CTA 0 of the head) the q rope pairs
    const int pos = __ldcg(a.pos);
    float cv[MAXR / AB_THREADS];
#pragma unroll
    for (int k = 0; k < MAXR / AB_THREADS; k++) {
        const int j = tid + AB_THREADS * k;
        cv[k] = j < a.kv_rank ? __ldcg(a.c + j) : 0.0f;
    }
    const float qn = tid < a.qk_nope ? __ldcg(a.q + (size_t)h * qk_per + tid) : 0.0f;
    const bool qrope = p == 0 && tid < a.qk_rope / 2;
    float x0 = 0.0f, x1 = 0.0f;
    if (qrope) {
        x0 = __ldcg(a.q + (size_t)h * qk_per + a.qk_nope + 2 * tid);
        x1 = __ldcg(a.q + (size_t)h * qk_per + a.qk_nope + 2 * tid + 1);
    }
    if (pos < 0 || pos >= a.ctx) {
        if (p == 0 && h == 0 && tid == 0) set_dev_error(0x81u);
        return;
    }
#pragma unroll
    for (int k = 0; k < MAXR / AB_THREADS; k++) {
        const int j = tid + AB_THREADS * k;
        if (j < a.kv_rank) {
            const uint16_t hb = f32_to_f16_ref(cv[k]);
            cs[j] = f16_to_f32(hb);
            if (h == 0 && (j >> 6) == p) a.latent[(size_t)pos * a.kv_rank + j] = hb;
        }
    }
    if (tid < a.qk_nope) qs[tid] = qn;
    if (qrope) {  // roped q slice (pairs 2i, 2i + 1)
        const float freq = powf(a.theta, -2.0f * (float)tid / (float)a.qk_rope);
        const float ang = (float)pos * freq, sn = sinf(ang), cs_ = cosf(ang);
        a.qr[(size_t)h * a.qk_rope + 2 * tid] = x0 * cs_ - x1 * sn;
        a.qr[(size_t)h * a.qk_rope + 2 * tid + 1] = x0 * sn + x1 * cs_;
    }
    __syncthreads();
    // absorbed query: qt[j] = sum_i W_kn[i][j] * q_nope[i]
    float lo[4] = {0.0f, 0.0f, 0.0f, 0.0f}, hi[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int k = 0; k < AB_ROWS; k++) {
        const int r = r0 + AB_RG * k;
        if (r < a.qk_nope) {
            const float qv = qs[r];
            float ds0, dm0, ds1, dm1;
            q4k_sub(hd[k], 2 * pair, ds0, dm0);
            q4k_sub(hd[k], 2 * pair + 1, ds1, dm1);
#pragma unroll
            for (int n = 0; n < 4; n++) {
                const unsigned byte = (cw[k] >> (8 * n)) & 255u;
                lo[n] += (ds0 * (float)(byte & 15u) - dm0) * qv;
                hi[n] += (ds1 * (float)(byte >> 4) - dm1) * qv;
            }
        }
    }
#pragma unroll
    for (int n = 0; n < 4; n++) {
#pragma unroll
        for (int o = 8; o <= 16; o <<= 1) {
            lo[n] += __shfl_xor_sync(0xffffffffu, lo[n], o);
            hi[n] += __shfl_xor_sync(0xffffffffu, hi[n], o);
        }
    }
    if (lane < 8) {
#pragma unroll
        for (int n = 0; n < 4; n++) red[warp][4 * w4 + n] = lo[n], red[warp][32 + 4 * w4 + n] = hi[n];
    }
    // rope keys of kv head h: rows of W_kr times the latent row as the cache holds it (f16)
    if (rope) {
        for (int i = rw0; i < rhi - rlo; i += 8) {
            if (i >= 8 && rlane) {
                const uint8_t *blk = WR + (size_t)(a.qk_nope + rlo + i) * rb + (t8 >> 4) * 144;
                rh = __ldg(reinterpret_cast<const uint4 *>(blk));
                rc = __ldg(reinterpret_cast<const uint2 *>(blk + 16 + 8 * (t8 & 15)));
            }
            float acc = 0.0f;
            if (rlane) {
                const int c8 = t8 & 15, pr = c8 >> 2;
                const int col = (t8 >> 4) * 256 + pr * 64 + 8 * (c8 & 3);
                float ds0, dm0, ds1, dm1;
                q4k_sub(rh, 2 * pr, ds0, dm0);
                q4k_sub(rh, 2 * pr + 1, ds1, dm1);
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const unsigned byte = ((e < 4 ? rc.x : rc.y) >> (8 * (e & 3))) & 255u;
                    acc += (ds0 * (float)(byte & 15u) - dm0) * cs[col + e];
                    acc += (ds1 * (float)(byte >> 4) - dm1) * cs[col + 32 + e];
                }
            }
            acc = warp_sum(acc);
            if (lane == 0) krp[warp >> 3][i] = acc;
        }
    }
    __syncthreads();
    if (tid < 64) {
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < AB_WARPS; w++) v += red[w][tid];
        a.qt[(size_t)h * a.kv_rank + b * 256 + pair * 64 + tid] = v;
    }
    if (rope) {
        for (int i = tid; i < (rhi - rlo) / 2; i += AB_THREADS) {
            const int g = rlo / 2 + i;  // pair index within the rope slice
            const float freq = powf(a.theta, -2.0f * (float)g / (float)a.qk_rope);
            const float ang = (float)pos * freq, sn = sinf(ang), cs_ = cosf(ang);
            const float k0 = krp[0][2 * i] + krp[1][2 * i], k1 = krp[0][2 * i + 1] + krp[1][2 * i + 1];
            float *dst = a.krope + ((size_t)pos * a.kv_heads + h) * a.qk_rope + 2 * g;
            dst[0] = k0 * cs_ - k1 * sn;
            dst[1] = k0 * sn + k1 * cs_;
        }
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

// ---------------------------------------------------------------- tensor-core form
// The same attention for kv_rank = 512 (DeepSeek-V2-Lite's latent) on the tensor cores,
// as the GQA kernel does it (decode_ops.cuh): the CTAs of one 16-CTA cluster take spans of
// the positions (att_span); latent sub-chunks of 32 rows arrive by TMA (eight 32 x 64 tiles,
// 128-byte swizzle) into two buffers; the main score term qt_h . c_t and the update
// cbar_h += sum_t p_t c_t are mma.sync.m16n8k16 with the 16 heads as the M rows, qt and P
// split into f16 hi + lo parts (c_t is f16 already); the rope term qr_h . kr_t (f32 keys)
// runs on the CUDA cores; spans merge through the cluster's shared memory.
constexpr int TC_R = 512;
constexpr int TC_T = 32;  // positions per sub-chunk

struct TcArgs {
    CUtensorMap lmap;  // latent [ctx][512] u16, box 32 rows x 64 dims, 128-byte swizzle
    const uint16_t *latent;  // the same rows (row pos is read again after the dependency wait)
    const float *qt;   // [heads][512]
    const float *qr;   // [heads][qk_rope]
    const float *krope;
    float *cbar;
    const int *pos;
    int heads, kv_heads, qk_rope, ctx;
    float scale;
};

struct TcSmem {
    uint8_t lb[2][TC_R / 64][TC_T * 128];  // [buffer][64-dim box]: 32 rows x 128 B, swizzled
    uint16_t qh[MAXH][TC_R + 8], ql[MAXH][TC_R + 8];
    uint16_t ph[MAXH][TC_T + 8], pl[MAXH][TC_T + 8];
    float qr[MAXH][MAXRP];
    float sc[2][MAXH][TC_T];  // main term, latent dims 0-255 / 256-511
    float sr[MAXH][TC_T];     // rope term
    float racc[ATT_SPANS][MAXH * TC_R / ATT_SPANS];
    float rm[ATT_SPANS][MAXH], rl[ATT_SPANS][MAXH];
    float mw[ATT_SPANS][MAXH], minv[MAXH];  // merge: weight of span cc for head j, 1 / sum
    float m[MAXH], l[MAXH], f[MAXH];
    uint64_t bar[2];
};

constexpr int TC_KR4 = 16;  // rope-key float4s per row held in registers (all of qk_rope <= 64)

__device__ __forceinline__ void cluster_st_f32x4(const void *p, int rank, float4 v)
{
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(tcmv::smem_u32(p)), "r"(rank));
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(ra), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// Address of dims d0..d0+7 (d0 a multiple of 8) of sub-chunk row `row`.
__device__ __forceinline__ const uint8_t *tc_at(const uint8_t (*buf)[TC_T * 128], int row, int d0)
{
    return buf[d0 >> 6] + att_swz(row, (d0 & 63) >> 3);
}

__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void *p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(tcmv::smem_u32(p)));
}

// Everything that does not come from the previous kernel is requested before the dependency
// wait: the latent sub-chunks (TMA) and the first sub-chunk's rope keys (registers) -- rows
// before pos were appended by earlier tokens, which completed before this token's kernels
// started.  Row pos itself is appended by the previous kernel: the CTA holding it loads the
// row again after the wait and writes it over what the prefetch saw (latent tile in shared
// memory, rope-key registers).
__global__ void __launch_bounds__(THREADS, 1) attn_tc_kernel(const __grid_constant__ TcArgs a)
{
    extern __shared__ __align__(1024) uint8_t tc_raw[];
    TcSmem &s = *reinterpret_cast<TcSmem *>(tc_raw + ((1024u - (tcmv::smem_u32(tc_raw) & 1023u)) & 1023u));
    const int H = a.heads, group = a.heads / a.kv_heads, RP = a.qk_rope;
    const int c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g8 = lane >> 2, t4 = lane & 3;
    const int pos = __ldcg(a.pos), seq = pos + 1;
    if (pos < 0 || seq > a.ctx) {  // the same for every CTA: all leave
        if (c == 0 && tid == 0) set_dev_error(0x82u);
        return;
    }
    const int span = att_span(seq), nch = (seq + span - 1) / span;
    const bool active = c < nch;
    const int tb = c * span, te = active ? min(seq, tb + span) : tb;
    const int nsub = active ? (te - tb + TC_T - 1) / TC_T : 0;
    const bool late = c == nch - 1;  // holds row pos, which the previous kernel appends
    if (nch == 1 && !active) return;
    griddep_launch();
    if (nch > 1) cluster_arrive_relaxed();
    if (tid == 0) {
        tcmv::mbar_init(&s.bar[0], 1);
        tcmv::mbar_init(&s.bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = tid; i < (MAXH - H) * (TC_R + 8); i += THREADS) (&s.qh[H][0])[i] = 0, (&s.ql[H][0])[i] = 0;
    for (int i = tid; i < (MAXH - H) * (TC_T + 8); i += THREADS) (&s.ph[H][0])[i] = 0, (&s.pl[H][0])[i] = 0;
    if (tid < MAXH) s.m[tid] = -INFINITY, s.l[tid] = 0.0f, s.f[tid] = 0.0f;
    __syncthreads();
    auto issue = [&](int i) {  // thread 0: rows t0.. of sub-chunk i into buffer i & 1
        const int t0 = tb + i * TC_T, b = i & 1;
        tcmv::mbar_expect_tx_arrive(&s.bar[b], (unsigned)(TC_R / 64) * TC_T * 128);
        for (int q = 0; q < TC_R / 64; q++) tma_tile_2d(s.lb[b][q], &a.lmap, 64 * q, t0, &s.bar[b]);
    };
    if (tid == 0) {
        if (nsub > 0) issue(0);
        if (nsub > 1) issue(1);
    }
    // rope keys: thread -> head rh, positions rt and rt + 16 of a sub-chunk; kreg holds the
    // first TC_KR4 float4s of each of the two rows (L2 loads: row pos is reloaded below)
    const int rh = tid >> 4, rt = tid & 15;
    float4 kreg[2][TC_KR4];
#define SB_KR_LOAD(T0, TN)                                                                          \
    _Pragma("unroll") for (int k = 0; k < 2; k++) {                                                 \
        if (rh < H && rt + 16 * k < (TN)) {                                                         \
            const float4 *kp = reinterpret_cast<const float4 *>(                                   \
                a.krope + ((size_t)((T0) + rt + 16 * k) * a.kv_heads + rh / group) * RP);          \
            _Pragma("unroll") for (int j = 0; j < TC_KR4; j++) if (4 * j < RP) kreg[k][j] = __ldcg(kp + j); \
        }                                                                                           \
    }
    if (nsub > 0) SB_KR_LOAD(tb, min(TC_T, te - tb))
    griddep_wait();  // qt, qr, this token's latent row and rope keys come from the previous kernel
    uint4 prow = make_uint4(0u, 0u, 0u, 0u);
    if (active && late) {
        if (tid < TC_R / 8) prow = __ldcg(reinterpret_cast<const uint4 *>(a.latent + (size_t)pos * TC_R) + tid);
        const int tp = pos - tb;  // the prefetched rope row of position pos, if sub-chunk 0 holds it
#pragma unroll
        for (int k = 0; k < 2; k++) {
            if (rh < H && tp == rt + 16 * k) {
                const float4 *kp =
                    reinterpret_cast<const float4 *>(a.krope + ((size_t)pos * a.kv_heads + rh / group) * RP);
#pragma unroll
                for (int j = 0; j < TC_KR4; j++)
                    if (4 * j < RP) kreg[k][j] = __ldcg(kp + j);
            }
        }
    }
    int issued = nsub < 2 ? nsub : 2;
    if (active) {
        float4 qv[(MAXH * TC_R / 4 + THREADS - 1) / THREADS], rv[(MAXH * MAXRP / 4 + THREADS - 1) / THREADS];
        const float4 *q4 = reinterpret_cast<const float4 *>(a.qt), *r4 = reinterpret_cast<const float4 *>(a.qr);
#pragma unroll
        for (int k = 0; k < (MAXH * TC_R / 4 + THREADS - 1) / THREADS; k++)
            if (tid + THREADS * k < H * TC_R / 4) qv[k] = __ldcg(q4 + tid + THREADS * k);
#pragma unroll
        for (int k = 0; k < (MAXH * MAXRP / 4 + THREADS - 1) / THREADS; k++)
            if (tid + THREADS * k < H * RP / 4) rv[k] = __ldcg(r4 + tid + THREADS * k);
#pragma unroll
        for (int k = 0; k < (MAXH * TC_R / 4 + THREADS - 1) / THREADS; k++) {
            const int i = tid + THREADS * k;
            if (i < H * TC_R / 4) {
                const int h = i / (TC_R / 4), d = 4 * (i % (TC_R / 4));
                split_f16(qv[k].x, s.qh[h][d], s.ql[h][d]);
                split_f16(qv[k].y, s.qh[h][d + 1], s.ql[h][d + 1]);
                split_f16(qv[k].z, s.qh[h][d + 2], s.ql[h][d + 2]);
                split_f16(qv[k].w, s.qh[h][d + 3], s.ql[h][d + 3]);
            }
        }
#pragma unroll
        for (int k = 0; k < (MAXH * MAXRP / 4 + THREADS - 1) / THREADS; k++) {
            const int i = tid + THREADS * k;
            if (i < H * RP / 4) {
                const int h = (4 * i) / RP, d = (4 * i) % RP;
                s.qr[h][d] = rv[k].x, s.qr[h][d + 1] = rv[k].y, s.qr[h][d + 2] = rv[k].z, s.qr[h][d + 3] = rv[k].w;
            }
        }
    }
    __syncthreads();
    float acc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
    const int mi = lane >> 3, mr = lane & 7;
    bool failed = false;
    int done = 0;
    for (int i = 0; i < nsub; i++) {
        const int t0 = tb + i * TC_T, tn = min(TC_T, te - t0), b = i & 1;
        // rope term from the registers (f32 keys): s.sr[head][position]
        if (rh < H) {
            const float *q = s.qr[rh];
#pragma unroll
            for (int k = 0; k < 2; k++) {
                const int t = rt + 16 * k;
                float r = 0.0f;
                if (t < tn) {
#pragma unroll
                    for (int j = 0; j < TC_KR4; j++)
                        if (4 * j < RP) {
                            const float4 kv = kreg[k][j];
                            r += q[4 * j] * kv.x + q[4 * j + 1] * kv.y + q[4 * j + 2] * kv.z + q[4 * j + 3] * kv.w;
                        }
                    const float4 *kp =
                        reinterpret_cast<const float4 *>(a.krope + ((size_t)(t0 + t) * a.kv_heads + rh / group) * RP);
                    for (int j = TC_KR4; 4 * j < RP; j++) {
                        const float4 kv = __ldcg(kp + j);
                        r += q[4 * j] * kv.x + q[4 * j + 1] * kv.y + q[4 * j + 2] * kv.z + q[4 * j + 3] * kv.w;
                    }
                }
                s.sr[rh][t] = r;
            }
        }
        // the next sub-chunk's keys: in flight during this one's tensor-core work
        if (i + 1 < nsub) SB_KR_LOAD(t0 + TC_T, min(TC_T, te - t0 - TC_T))
        if (!tcmv::mbar_wait(&s.bar[b], (unsigned)(i >> 1) & 1u)) failed = true;
        if (__syncthreads_or(failed)) {
            failed = true;
            break;
        }
        done = i + 1;
        // rows past the sub-chunk: zero (P is zero there; other rows could hold non-finite values)
        for (int idx = tid; idx < (TC_T - tn) * (TC_R / 2); idx += THREADS) {
            const int r = tn + idx / (TC_R / 2), w = idx % (TC_R / 2);
            reinterpret_cast<uint32_t *>(s.lb[b][w >> 5] + r * 128)[w & 31] = 0u;
        }
        // row pos as the previous kernel wrote it (dims 8 tid .. 8 tid + 7)
        if (late && tid < TC_R / 8 && pos >= t0 && pos < t0 + tn)
            *reinterpret_cast<uint4 *>(s.lb[b][tid >> 3] + att_swz(pos - t0, tid & 7)) = prow;
        __syncthreads();
        // main term: warp w takes positions 8(w & 3) .. +8 and latent dims 256(w >> 2) .. +256
        {
            const int n0 = 8 * (warp & 3), kh = warp >> 2;
            float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (n0 < tn) {
#pragma unroll 4
                for (int ks = 0; ks < 16; ks++) {
                    const int k0 = kh * 256 + ks * 16;
                    uint32_t ah[4], al[4], bf[2];
                    ldsm_x4(ah, &s.qh[(mi & 1) * 8 + mr][k0 + (mi >> 1) * 8]);
                    ldsm_x4(al, &s.ql[(mi & 1) * 8 + mr][k0 + (mi >> 1) * 8]);
                    ldsm_x2(bf, tc_at(s.lb[b], n0 + mr, k0 + ((lane >> 3) & 1) * 8));
                    tcmv::mma_f16(d, ah[0], ah[1], ah[2], ah[3], bf[0], bf[1]);
                    tcmv::mma_f16(d, al[0], al[1], al[2], al[3], bf[0], bf[1]);
                }
            }
            // d: (head g8 | g8 + 8) x (position n0 + 2 t4 | + 1)
            s.sc[kh][g8][n0 + 2 * t4] = d[0];
            s.sc[kh][g8][n0 + 2 * t4 + 1] = d[1];
            s.sc[kh][g8 + 8][n0 + 2 * t4] = d[2];
            s.sc[kh][g8 + 8][n0 + 2 * t4 + 1] = d[3];
        }
        __syncthreads();
        // online softmax: warp w takes heads w and w + 8, lane = position
        for (int hh = warp; hh < H; hh += THREADS / 32) {
            const float sv = lane < tn ? ((s.sc[0][hh][lane] + s.sc[1][hh][lane]) + s.sr[hh][lane]) * a.scale : -INFINITY;
            float mx = sv;
#pragma unroll
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float mo = s.m[hh], mn = fmaxf(mo, mx);
            const float p = lane < tn ? expf(sv - mn) : 0.0f;
            split_f16(p, s.ph[hh][lane], s.pl[hh][lane]);
            const float l = warp_sum(p);
            if (lane == 0) {
                const float f = mo == -INFINITY ? 0.0f : expf(mo - mn);
                s.f[hh] = f;
                s.l[hh] = s.l[hh] * f + l;
                s.m[hh] = mn;
            }
        }
        __syncthreads();
        // cbar (heads x dims) = f * cbar + P . C: warp w takes latent dims 64w .. 64w + 63
        {
            const float fa = s.f[g8], fb = s.f[g8 + 8];
#pragma unroll
            for (int nt = 0; nt < 8; nt++) acc[nt][0] *= fa, acc[nt][1] *= fa, acc[nt][2] *= fb, acc[nt][3] *= fb;
            for (int k0 = 0; k0 < tn; k0 += 16) {
                uint32_t ph[4], pl[4];
                ldsm_x4(ph, &s.ph[(mi & 1) * 8 + mr][k0 + (mi >> 1) * 8]);
                ldsm_x4(pl, &s.pl[(mi & 1) * 8 + mr][k0 + (mi >> 1) * 8]);
#pragma unroll
                for (int nt = 0; nt < 8; nt += 2) {
                    const int n0 = warp * 64 + nt * 8;
                    uint32_t bt[4];
                    ldsm_x4_t(bt, tc_at(s.lb[b], k0 + (mi & 1) * 8 + mr, n0 + (mi >> 1) * 8));
                    tcmv::mma_f16(acc[nt], ph[0], ph[1], ph[2], ph[3], bt[0], bt[1]);
                    tcmv::mma_f16(acc[nt], pl[0], pl[1], pl[2], pl[3], bt[0], bt[1]);
                    tcmv::mma_f16(acc[nt + 1], ph[0], ph[1], ph[2], ph[3], bt[2], bt[3]);
                    tcmv::mma_f16(acc[nt + 1], pl[0], pl[1], pl[2], pl[3], bt[2], bt[3]);
                }
            }
        }
        __syncthreads();  // buffer b, the scores and P are free again
        if (tid == 0 && i + 2 < nsub) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(i + 2);
        }
        if (i + 2 < nsub) issued = i + 3;
    }
#undef SB_KR_LOAD
    if (failed) {
        if (tid == 0) {
            set_dev_error(0x83u);
            for (int i = done; i < issued; i++) tcmv::mbar_wait(&s.bar[i & 1], (unsigned)(i >> 1) & 1u);
        }
        __syncthreads();
    }
    if (nch == 1) {  // the whole context in one span: normalise and store
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            const int d = warp * 64 + nt * 8 + 2 * t4;
#pragma unroll
            for (int hb = 0; hb < 2; hb++) {
                const int h = g8 + 8 * hb;
                if (h >= H) continue;
                const float l = s.l[h], r = l > 0.0f ? 1.0f / l : 0.0f;
                a.cbar[(size_t)h * TC_R + d] = l > 0.0f ? acc[nt][2 * hb] * r : 0.0f;
                a.cbar[(size_t)h * TC_R + d + 1] = l > 0.0f ? acc[nt][2 * hb + 1] * r : 0.0f;
            }
        }
        return;
    }
    // merge the spans (combinar_trozos): CTA r forms outputs r*per .. (o = head * 512 + dim).
    // The partial sums go through latent buffer 0 (free after the loop) first, so that each
    // warp's push is 512 contiguous bytes into one CTA (a fragment spans 8 heads: 8 CTAs).
    const int per = H * TC_R / ATT_SPANS;
    float *stage = reinterpret_cast<float *>(&s.lb[0][0][0]);
    static_assert(sizeof(s.lb[0]) >= MAXH * TC_R * 4, "partial sums fit one latent buffer");
    if (active) {
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int hb = 0; hb < 2; hb++) {
                const int h = g8 + 8 * hb, d = warp * 64 + nt * 8 + 2 * t4;
                if (h < H)
                    *reinterpret_cast<float2 *>(stage + h * TC_R + d) = make_float2(acc[nt][2 * hb], acc[nt][2 * hb + 1]);
            }
    }
    __syncthreads();
    cluster_wait();
    if (active) {
        const int per4 = per / 4;
        for (int f = tid; f < H * TC_R / 4; f += THREADS) {
            const int r = f / per4, q = f - r * per4;
            cluster_st_f32x4(&s.racc[c][4 * q], r, *reinterpret_cast<const float4 *>(stage + 4 * f));
        }
        if (tid < ATT_SPANS * H) {
            const int r = tid / H, j = tid % H;
            cluster_st_f32(&s.rm[c][j], r, s.m[j]);
            cluster_st_f32(&s.rl[c][j], r, s.l[j]);
        }
    }
    cluster_sync();
    {  // thread (head j, span cc): the span weight exp(m_cc - M) and 1 / sum_cc weight * l_cc,
       // max and sum over the 16 spans of a half-warp by shuffles
        static_assert(MAXH * ATT_SPANS == THREADS, "one thread per (head, span)");
        const int j = tid >> 4, cc = tid & 15;
        const bool ok = j < H && cc < nch && s.rl[cc][j] > 0.0f;
        const float lv = ok ? s.rl[cc][j] : 0.0f, mv = ok ? s.rm[cc][j] : -INFINITY;
        float M = mv;
#pragma unroll
        for (int o = 8; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float w = ok ? expf(mv - M) : 0.0f;
        float L = w * lv;
#pragma unroll
        for (int o = 8; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        if (j < H) {
            s.mw[cc][j] = w;
            if (cc == 0) s.minv[j] = L > 0.0f ? 1.0f / L : 0.0f;
        }
    }
    __syncthreads();
    for (int q = tid; q < per; q += THREADS) {
        const int o = c * per + q, j = o / TC_R;
        float O = 0.0f;
        for (int cc = 0; cc < nch; cc++) O += s.mw[cc][j] * s.racc[cc][q];
        a.cbar[o] = s.minv[j] > 0.0f ? O * s.minv[j] : 0.0f;
    }
}

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
        qk_nope > AB_RG * AB_ROWS || !qk_rope || qk_rope % 2 || qk_rope > MAXRP || !ctx)
        return -1;
    if (((uintptr_t)k_up) & 15) return -2;
    AbsorbArgs a{q, c, (const uint8_t *)k_up, latent, krope, qt, qr, pos, (int)heads, (int)kv_heads, (int)kv_rank,
                 (int)qk_nope, (int)qk_rope, (int)ctx, theta};
    return sb::launch_k(absorb_kernel, dim3((unsigned)(kv_rank / 64), (unsigned)heads), dim3(AB_THREADS), 0, pdl,
                        (cudaStream_t)stream, a);
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
    if (kv_rank == TC_R && qk_rope % 4 == 0 && !(((uintptr_t)qt | (uintptr_t)qr | (uintptr_t)krope) & 15)) {
        // the tensor-core form: one cluster of ATT_SPANS CTAs (a non-portable cluster size)
        static size_t tc_rec[64];
        static std::mutex mu;
        {
            std::lock_guard<std::mutex> lk(mu);
            int dev = 0;
            cudaGetDevice(&dev);
            if (dev < 0 || dev >= 64) return -3;
            if (!tc_rec[dev]) {
                if (cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(TcSmem) + 1024) != cudaSuccess ||
                    cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
                        cudaSuccess)
                    return -3;
                tc_rec[dev] = 1;
            }
        }
        TcArgs t{};
        {
            sb::tcmv::EncodeTiledFn fn = sb::tcmv::encode_fn();
            if (!fn) return -6;
            cuuint64_t dims[2] = {(cuuint64_t)TC_R, (cuuint64_t)ctx};
            cuuint64_t strides[1] = {(cuuint64_t)TC_R * 2};
            cuuint32_t box[2] = {64, (cuuint32_t)TC_T};
            cuuint32_t es[2] = {1, 1};
            if (fn(&t.lmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t *>(latent), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                return -7;
        }
        t.latent = latent, t.qt = qt, t.qr = qr, t.krope = krope, t.cbar = cbar, t.pos = pos;
        t.heads = (int)heads, t.kv_heads = (int)kv_heads, t.qk_rope = (int)qk_rope, t.ctx = (int)ctx;
        t.scale = 1.0f / sqrtf((float)(qk_nope + qk_rope));
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3((unsigned)sb::ATT_SPANS);
        lc.blockDim = dim3(THREADS);
        lc.dynamicSmemBytes = sizeof(TcSmem) + 1024;
        lc.stream = (cudaStream_t)stream;
        cudaLaunchAttribute at[2];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = sb::ATT_SPANS, at[0].val.clusterDim.y = 1, at[0].val.clusterDim.z = 1;
        at[1] = sb::pdl_attr();
        lc.attrs = at;
        lc.numAttrs = pdl ? 2 : 1;
        return cudaLaunchKernelEx(&lc, attn_tc_kernel, t) == cudaSuccess ? 0 : -4;
    }
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
