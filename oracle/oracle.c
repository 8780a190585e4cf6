/*
 * oracle.c -- CPU restatement of demonodojo/soso's quantized decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA kernels in
 * soso_b200/csrc.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load it.  The product library
 * (libsosob200.so) never links, loads or calls anything in oracle/.
 *
 * Every function restates one reference function, in the reference's own
 * order of floating-point operations, and names the file:line it follows
 * (paths are relative to the demonodojo/soso checkout).  The reference is
 * Rust and cannot be compiled in this image (no cargo/rustc), so the
 * restatement is pinned instead against:
 *   - the golden vectors of crates/sosomodel/tests/dequant_golden.rs:44-114
 *     (Q4_K 6-bit scale table, Q4_K block dot -15.875, .som Q8_0 dot
 *     172.59375) and crates/gguf2som/src/lib.rs:1866-1889 (Q6_K -1.0 block);
 *   - lxdde/ports/nouveau/q4k_decode.h, the reference's own plain-C decoder,
 *     compiled from its source into oracle/_ref/ by oracle/Makefile.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

#define OR_API __attribute__((visibility("default")))

/* sosomodel dtype codes, crates/sosomodel/src/layout.rs:8-12.  13 (Q6_K, GGML
 * layout, 210 B / 256 weights) is not a reference dtype: the reference converts
 * Q6_K to Q8_0 on import (crates/gguf2som/src/lib.rs:1592-1610).  It is this
 * project's extension for a native Q6_K matvec. */
enum { OR_F32 = 1, OR_Q8_0 = 2, OR_Q4_K = 3, OR_Q6_K = 13 };

/* ---------------------------------------------------------------- f16 ---- */

/* crates/sosomodel/src/dequant.rs:26-45 (f16_to_f32, incl. subnormals). */
OR_API float or_f16_to_f32(uint16_t bits)
{
    uint32_t sign = (bits >> 15) & 1u, exp = (bits >> 10) & 0x1fu, frac = bits & 0x3ffu;
    union { uint32_t u; float f; } c;
    if (exp == 0) {
        if (frac == 0) { c.u = sign << 31; return c.f; }
        float v = ((float)frac / 1024.0f) * 6.1035156e-5f;
        return sign ? -v : v;
    }
    if (exp == 31) {
        if (frac == 0) { c.u = (sign << 31) | 0x7f800000u; return c.f; }
        return NAN;
    }
    c.u = (sign << 31) | ((exp + 112u) << 23) | (frac << 13);
    return c.f;
}

/* crates/soso-llm-core/src/f16.rs:10-37 (round to nearest, ties up). */
OR_API uint16_t or_f32_to_f16(float v)
{
    union { float f; uint32_t u; } c = { v };
    uint32_t bits = c.u;
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int32_t exp = (int32_t)((bits >> 23) & 0xffu);
    uint32_t frac = bits & 0x7fffffu;
    if (exp == 255) return (uint16_t)(sign | 0x7c00u | (frac ? 0x200u : 0u));
    int32_t e = exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t f = frac | 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint16_t sub = (uint16_t)(f >> shift);
        uint16_t round = (uint16_t)((f >> (shift - 1)) & 1u);
        return (uint16_t)(sign | (uint16_t)(sub + round));
    }
    uint32_t half = ((uint32_t)e << 10) | (frac >> 13);
    uint16_t round = (uint16_t)((frac >> 12) & 1u);
    return (uint16_t)((uint16_t)(sign | (uint16_t)half) + round);
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline float rdf32(const uint8_t *p) { float f; memcpy(&f, p, 4); return f; }

/* ------------------------------------------------------------ layout ---- */

/* crates/sosomodel/src/dequant.rs:53-63 (row_bytes); 0 = None. */
OR_API size_t or_row_bytes(uint8_t dtype, size_t cols)
{
    size_t elems, bytes;
    switch (dtype) {
    case OR_Q8_0: elems = 32; bytes = 36; break;   /* layout.rs:57-59 */
    case OR_Q4_K: elems = 256; bytes = 144; break;  /* layout.rs:63-64 */
    case OR_Q6_K: elems = 256; bytes = 210; break;  /* GGML block_q6_K */
    case OR_F32: return cols * 4;
    default: return 0;
    }
    if (cols == 0 || cols % elems) return 0;
    return cols / elems * bytes;
}

/* ------------------------------------------------------------- Q4_K ---- */

/* crates/sosomodel/src/dequant.rs:150-167 (get_scale_min_k4). */
OR_API void or_q4k_scale_min(const uint8_t *s, int j, uint8_t *sc, uint8_t *m)
{
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* crates/sosomodel/src/dequant.rs:172-191 (q4k_dot_sub). */
OR_API float or_q4k_dot_sub(const uint8_t *blk, int j, const float *x)
{
    float d = or_f16_to_f32(rd16(blk)), dmin = or_f16_to_f32(rd16(blk + 2));
    uint8_t sc, m;
    or_q4k_scale_min(blk + 4, j, &sc, &m);
    const uint8_t *qs = blk + 16;
    int pair = j >> 1, alto = j & 1;
    float qx = 0.0f, sx = 0.0f;
    for (int l = 0; l < 32; l++) {
        uint8_t q = qs[pair * 32 + l];
        float v = (float)(alto ? (q >> 4) : (q & 0x0F));
        qx += v * x[l];
        sx += x[l];
    }
    return (d * (float)sc) * qx - (dmin * (float)m) * sx;
}

/* crates/sosomodel/src/dequant.rs:195-201 (q4k_dot_ref). */
OR_API float or_q4k_dot_ref(const uint8_t *blk, const float *x)
{
    float acc = 0.0f;
    for (int j = 0; j < 8; j++) acc += or_q4k_dot_sub(blk, j, x + j * 32);
    return acc;
}

/* crates/sosomodel/src/dequant.rs:204-241 (dequant_q4_k_range, whole tensor). */
OR_API int or_dequant_q4_k(const uint8_t *bytes, size_t nbytes, float *out, size_t n)
{
    if (nbytes % 144 || n != nbytes / 144 * 256) return -1;
    for (size_t b = 0; b < nbytes / 144; b++) {
        const uint8_t *blk = bytes + b * 144;
        float d = or_f16_to_f32(rd16(blk)), dmin = or_f16_to_f32(rd16(blk + 2));
        const uint8_t *qs = blk + 16;
        for (int pair = 0; pair < 4; pair++) {
            uint8_t sc1, m1, sc2, m2;
            or_q4k_scale_min(blk + 4, 2 * pair, &sc1, &m1);
            or_q4k_scale_min(blk + 4, 2 * pair + 1, &sc2, &m2);
            float d1 = d * (float)sc1, min1 = dmin * (float)m1;
            float d2 = d * (float)sc2, min2 = dmin * (float)m2;
            float *o = out + b * 256 + pair * 64;
            for (int l = 0; l < 32; l++) {
                uint8_t q = qs[pair * 32 + l];
                o[l] = d1 * (float)(q & 0x0F) - min1;
                o[32 + l] = d2 * (float)(q >> 4) - min2;
            }
        }
    }
    return 0;
}

/* crates/soso-llm-core/src/gemm.rs:428-461 (matvec_q4_k_scalar). */
OR_API int or_matvec_q4_k(const uint8_t *bytes, size_t rows, size_t cols, const float *x, float *out)
{
    size_t rb = or_row_bytes(OR_Q4_K, cols);
    if (!rb) return -1;
    for (size_t r = 0; r < rows; r++) {
        const uint8_t *row = bytes + r * rb;
        float acc = 0.0f;
        for (size_t b = 0; b < cols / 256; b++) {
            const uint8_t *blk = row + b * 144;
            float d = or_f16_to_f32(rd16(blk)), dmin = or_f16_to_f32(rd16(blk + 2));
            const uint8_t *qs = blk + 16;
            const float *xb = x + b * 256;
            for (int pair = 0; pair < 4; pair++) {
                uint8_t sc1, m1, sc2, m2;
                or_q4k_scale_min(blk + 4, 2 * pair, &sc1, &m1);
                or_q4k_scale_min(blk + 4, 2 * pair + 1, &sc2, &m2);
                const float *x1 = xb + pair * 64, *x2 = xb + pair * 64 + 32;
                const uint8_t *q = qs + pair * 32;
                float s1 = 0, sx1 = 0, s2 = 0, sx2 = 0;
                for (int l = 0; l < 32; l++) {
                    s1 += (float)(q[l] & 0x0F) * x1[l];
                    sx1 += x1[l];
                    s2 += (float)(q[l] >> 4) * x2[l];
                    sx2 += x2[l];
                }
                acc += d * (float)sc1 * s1 - dmin * (float)m1 * sx1;
                acc += d * (float)sc2 * s2 - dmin * (float)m2 * sx2;
            }
        }
        out[r] = acc;
    }
    return 0;
}

/* ------------------------------------------------------------- Q8_0 ---- */

/* crates/sosomodel/src/dequant.rs:74-102 (.som Q8_0: f32 scale + 32 i8). */
OR_API int or_dequant_q8_0(const uint8_t *bytes, size_t nbytes, float *out, size_t n)
{
    if (nbytes % 36 || n != nbytes / 36 * 32) return -1;
    for (size_t b = 0; b < nbytes / 36; b++) {
        const uint8_t *c = bytes + b * 36;
        float scale = rdf32(c);
        for (int j = 0; j < 32; j++) out[b * 32 + j] = (float)(int8_t)c[4 + j] * scale;
    }
    return 0;
}

/* crates/soso-llm-core/src/gemm.rs:315-332 (matvec_q8_0_scalar). */
OR_API int or_matvec_q8_0(const uint8_t *bytes, size_t rows, size_t cols, const float *x, float *out)
{
    size_t rb = or_row_bytes(OR_Q8_0, cols);
    if (!rb) return -1;
    for (size_t r = 0; r < rows; r++) {
        const uint8_t *row = bytes + r * rb;
        float acc = 0.0f;
        for (size_t b = 0; b < cols / 32; b++) {
            const uint8_t *c = row + b * 36;
            float scale = rdf32(c), s = 0.0f;
            for (int j = 0; j < 32; j++) s += (float)(int8_t)c[4 + j] * x[b * 32 + j];
            acc += scale * s;
        }
        out[r] = acc;
    }
    return 0;
}

/* ------------------------------------------------------------- Q6_K ---- */

/* crates/gguf2som/src/lib.rs:1639-1661 (dequant_q6_k_block), one 210-B block. */
OR_API void or_dequant_q6_k_block(const uint8_t *blk, float *out)
{
    const uint8_t *ql0 = blk, *qh0 = blk + 128;
    const int8_t *sc0 = (const int8_t *)(blk + 192);
    float d = or_f16_to_f32(rd16(blk + 208));
    for (int n = 0; n < 2; n++) {
        const uint8_t *ql = ql0 + n * 64, *qh = qh0 + n * 32;
        const int8_t *sc = sc0 + n * 8;
        float *y = out + n * 128;
        for (int l = 0; l < 32; l++) {
            int is = l / 16;
            int q1 = (int)((ql[l] & 0x0F) | ((qh[l] & 3) << 4)) - 32;
            int q2 = (int)((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
            int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            y[l] = d * (float)sc[is] * (float)q1;
            y[l + 32] = d * (float)sc[is + 2] * (float)q2;
            y[l + 64] = d * (float)sc[is + 4] * (float)q3;
            y[l + 96] = d * (float)sc[is + 6] * (float)q4;
        }
    }
}

OR_API int or_dequant_q6_k(const uint8_t *bytes, size_t nbytes, float *out, size_t n)
{
    if (nbytes % 210 || n != nbytes / 210 * 256) return -1;
    for (size_t b = 0; b < nbytes / 210; b++) or_dequant_q6_k_block(bytes + b * 210, out + b * 256);
    return 0;
}

/* The reference has no Q6_K matvec.  Its generic path for GGML K-quants,
 * crates/soso-llm-core/src/gemm.rs matvec_iq (dequantize a row with
 * dequant_iq_range, then `acc += w * xi` in element order), is the order
 * followed here, with the Q6_K block decoder above. */
OR_API int or_matvec_q6_k(const uint8_t *bytes, size_t rows, size_t cols, const float *x, float *out)
{
    size_t rb = or_row_bytes(OR_Q6_K, cols);
    if (!rb) return -1;
    float *w = (float *)malloc(cols * sizeof(float));
    if (!w) return -2;
    for (size_t r = 0; r < rows; r++) {
        or_dequant_q6_k(bytes + r * rb, rb, w, cols);
        float acc = 0.0f;
        for (size_t c = 0; c < cols; c++) acc += w[c] * x[c];
        out[r] = acc;
    }
    free(w);
    return 0;
}

/* ---------------------------------------------------- dispatch + f64 ---- */

OR_API int or_dequant(uint8_t dtype, const uint8_t *bytes, size_t nbytes, float *out, size_t n)
{
    switch (dtype) {
    case OR_Q8_0: return or_dequant_q8_0(bytes, nbytes, out, n);
    case OR_Q4_K: return or_dequant_q4_k(bytes, nbytes, out, n);
    case OR_Q6_K: return or_dequant_q6_k(bytes, nbytes, out, n);
    case OR_F32:
        if (nbytes != n * 4) return -1;
        memcpy(out, bytes, nbytes);
        return 0;
    }
    return -1;
}

OR_API int or_matvec(uint8_t dtype, const uint8_t *bytes, size_t rows, size_t cols, const float *x, float *out)
{
    switch (dtype) {
    case OR_Q8_0: return or_matvec_q8_0(bytes, rows, cols, x, out);
    case OR_Q4_K: return or_matvec_q4_k(bytes, rows, cols, x, out);
    case OR_Q6_K: return or_matvec_q6_k(bytes, rows, cols, x, out);
    case OR_F32: {
        /* crates/soso-llm-core/src/gemm.rs matvec_f32_scalar */
        const float *m = (const float *)bytes;
        for (size_t r = 0; r < rows; r++) {
            float acc = 0.0f;
            for (size_t c = 0; c < cols; c++) acc += m[r * cols + c] * x[c];
            out[r] = acc;
        }
        return 0;
    }
    }
    return -1;
}

/* f64 "truth": dequantize each row exactly (the decoders above are exact in
 * f32 except for d*sc products, which are exact too for these formats' value
 * ranges) and accumulate in double, as crates/soso-llm-api/tests/cuda_matvec.rs
 * :35-84 does for its GPU parity reference. */
OR_API int or_matvec_f64(uint8_t dtype, const uint8_t *bytes, size_t rows, size_t cols,
                         const float *x, size_t n, double *out)
{
    size_t rb = or_row_bytes(dtype, cols);
    if (!rb) return -1;
    float *w = (float *)malloc(cols * sizeof(float));
    if (!w) return -2;
    for (size_t r = 0; r < rows; r++) {
        if (or_dequant(dtype, bytes + r * rb, rb, w, cols)) { free(w); return -1; }
        for (size_t t = 0; t < n; t++) {
            double s = 0.0;
            const float *xt = x + t * cols;
            for (size_t c = 0; c < cols; c++) s += (double)w[c] * (double)xt[c];
            out[t * rows + r] = s;
        }
    }
    free(w);
    return 0;
}

/* -------------------------------------------------------- quantizers ---- */

/* crates/soso-llm-core/src/quant.rs:8-24 (quantize_q8_0; last block zero-padded). */
OR_API void or_quantize_q8_0(const float *src, size_t n, uint8_t *out)
{
    size_t blocks = (n + 31) / 32;
    for (size_t b = 0; b < blocks; b++) {
        float mx = 0.0f;
        for (size_t i = 0; i < 32 && b * 32 + i < n; i++) mx = fmaxf(mx, fabsf(src[b * 32 + i]));
        float scale = mx > 0.0f ? mx / 127.0f : 1.0f;
        uint8_t *o = out + b * 36;
        memcpy(o, &scale, 4);
        for (size_t i = 0; i < 32; i++) {
            float v = b * 32 + i < n ? src[b * 32 + i] : 0.0f;
            float q = roundf(v / scale);
            if (q < -127.0f) q = -127.0f;
            if (q > 127.0f) q = 127.0f;
            o[4 + i] = (uint8_t)(int8_t)q;
        }
    }
}

/* crates/soso-llm-core/src/quant.rs:43-52 (q4k_pack_scales). */
static void q4k_pack_scales(const uint8_t sc[8], const uint8_t m[8], uint8_t s[12])
{
    for (int j = 0; j < 4; j++) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0x0F) | ((m[j + 4] & 0x0F) << 4));
    }
}

static uint8_t q4k_quantize_nibble(float v, float s, float o)
{
    if (s <= 0.0f) return 0;
    float q = roundf((v + o) / s);
    if (q < 0.0f) q = 0.0f;
    if (q > 15.0f) q = 15.0f;
    return (uint8_t)q;
}

/* crates/soso-llm-core/src/quant.rs:75-154 (quantize_q4_k). */
OR_API void or_quantize_q4_k(const float *src, size_t n, uint8_t *out)
{
    size_t blocks = (n + 255) / 256;
    for (size_t b = 0; b < blocks; b++) {
        size_t base = b * 256;
#define VAL(i) ((base + (i)) < n ? src[base + (i)] : 0.0f)
        float s_ideal[8], o_ideal[8];
        for (int j = 0; j < 8; j++) {
            float lo = 0.0f, hi = 0.0f;
            for (int l = 0; l < 32; l++) {
                float v = VAL(j * 32 + l);
                if (v < lo) lo = v;
                if (v > hi) hi = v;
            }
            s_ideal[j] = (hi - lo) / 15.0f;
            o_ideal[j] = -lo;
        }
        float max_s = 0.0f, max_o = 0.0f;
        for (int j = 0; j < 8; j++) {
            if (s_ideal[j] > max_s) max_s = s_ideal[j];
            if (o_ideal[j] > max_o) max_o = o_ideal[j];
        }
        uint16_t d_bits = or_f32_to_f16(max_s / 63.0f), dmin_bits = or_f32_to_f16(max_o / 63.0f);
        float d = or_f16_to_f32(d_bits), dmin = or_f16_to_f32(dmin_bits);
        uint8_t sc[8], m[8];
        for (int j = 0; j < 8; j++) {
            float a = d > 0.0f ? roundf(s_ideal[j] / d) : 0.0f;
            float c = dmin > 0.0f ? roundf(o_ideal[j] / dmin) : 0.0f;
            sc[j] = (uint8_t)(a < 0 ? 0 : a > 63 ? 63 : a);
            m[j] = (uint8_t)(c < 0 ? 0 : c > 63 ? 63 : c);
        }
        uint8_t *o = out + b * 144;
        o[0] = (uint8_t)d_bits; o[1] = (uint8_t)(d_bits >> 8);
        o[2] = (uint8_t)dmin_bits; o[3] = (uint8_t)(dmin_bits >> 8);
        q4k_pack_scales(sc, m, o + 4);
        for (int pair = 0; pair < 4; pair++) {
            float s1 = d * (float)sc[2 * pair], o1 = dmin * (float)m[2 * pair];
            float s2 = d * (float)sc[2 * pair + 1], o2 = dmin * (float)m[2 * pair + 1];
            for (int l = 0; l < 32; l++) {
                uint8_t q1 = q4k_quantize_nibble(VAL(pair * 64 + l), s1, o1);
                uint8_t q2 = q4k_quantize_nibble(VAL(pair * 64 + 32 + l), s2, o2);
                o[16 + pair * 32 + l] = (uint8_t)(q1 | (q2 << 4));
            }
        }
#undef VAL
    }
}

/* Q6_K quantizer (GGML block_q6_K layout, the inverse of the decoder above).
 * The reference has none (it only ever reads Q6_K to convert it to Q8_0), so
 * this is this project's own: per 16-element group an i8 scale relative to a
 * per-block f16 d, codes round((v / (d*sc))) + 32 clamped to [0, 63]. */
OR_API void or_quantize_q6_k(const float *src, size_t n, uint8_t *out)
{
    size_t blocks = (n + 255) / 256;
    for (size_t b = 0; b < blocks; b++) {
        float v[256];
        for (int i = 0; i < 256; i++) v[i] = b * 256 + i < n ? src[b * 256 + i] : 0.0f;
        float gscale[16], maxg = 0.0f;
        for (int g = 0; g < 16; g++) {
            float mx = 0.0f;
            for (int i = 0; i < 16; i++) mx = fmaxf(mx, fabsf(v[g * 16 + i]));
            gscale[g] = mx / 31.0f;
            if (gscale[g] > maxg) maxg = gscale[g];
        }
        uint16_t d_bits = or_f32_to_f16(maxg / 127.0f);
        float d = or_f16_to_f32(d_bits);
        int8_t sc[16];
        for (int g = 0; g < 16; g++) {
            float s = d > 0.0f ? roundf(gscale[g] / d) : 0.0f;
            if (s > 127.0f) s = 127.0f;
            sc[g] = (int8_t)s;
        }
        uint8_t q[256];
        for (int i = 0; i < 256; i++) {
            float ds = d * (float)sc[i / 16];
            float qq = ds > 0.0f ? roundf(v[i] / ds) + 32.0f : 32.0f;
            if (qq < 0.0f) qq = 0.0f;
            if (qq > 63.0f) qq = 63.0f;
            q[i] = (uint8_t)qq;
        }
        /* Inverse of dequant_q6_k_block's element mapping. */
        uint8_t *o = out + b * 210;
        memset(o, 0, 210);
        for (int nn = 0; nn < 2; nn++) {
            uint8_t *ql = o + nn * 64, *qh = o + 128 + nn * 32;
            const uint8_t *y = q + nn * 128;
            for (int l = 0; l < 32; l++) {
                ql[l] = (uint8_t)((y[l] & 15) | ((y[l + 64] & 15) << 4));
                ql[l + 32] = (uint8_t)((y[l + 32] & 15) | ((y[l + 96] & 15) << 4));
                qh[l] = (uint8_t)((y[l] >> 4) | ((y[l + 32] >> 4) << 2) | ((y[l + 64] >> 4) << 4) |
                                  ((y[l + 96] >> 4) << 6));
            }
        }
        memcpy(o + 192, sc, 16);
        o[208] = (uint8_t)d_bits;
        o[209] = (uint8_t)(d_bits >> 8);
    }
}

/* ------------------------------------------------------ float ops ---- */

/* crates/soso-llm-core/src/gemm.rs:93-100 (rmsnorm, in place). */
OR_API void or_rmsnorm(float *x, const float *w, size_t n, float eps)
{
    float var = 0.0f;
    for (size_t i = 0; i < n; i++) var += x[i] * x[i];
    var /= (float)n;
    float scale = 1.0f / sqrtf(var + eps);
    for (size_t i = 0; i < n; i++) x[i] = x[i] * scale * w[i];
}

/* crates/soso-llm-core/src/gemm.rs:1452-1491 (rope_cabezas): cos/sin per pair
 * once, applied to every head; NeoX pairs (i, i+half), else (2i, 2i+1). */
OR_API void or_rope_heads(float *x, size_t n_heads, size_t hd, size_t pos, float theta, int neox)
{
    size_t half = hd / 2;
    float cs[512], sn[512];
    if (hd < 2 || half > 512) return;
    for (size_t i = 0; i < half; i++) {
        float freq = powf(theta, -2.0f * (float)i / (float)hd);
        float ang = (float)pos * freq;
        sn[i] = sinf(ang);
        cs[i] = cosf(ang);
    }
    for (size_t h = 0; h < n_heads; h++) {
        float *v = x + h * hd;
        for (size_t i = 0; i < half; i++) {
            size_t a = neox ? i : 2 * i, b = neox ? i + half : 2 * i + 1;
            float va = v[a], vb = v[b];
            v[a] = va * cs[i] - vb * sn[i];
            v[b] = va * sn[i] + vb * cs[i];
        }
    }
}

/* crates/soso-llm-core/src/gemm.rs:1346 + :1500-1520 (rope_inplace_n: llama
 * pairs over the first n_rot elements, freq = theta^(-2i/n_rot)). */
OR_API void or_rope_llama_n(float *x, size_t pos, float theta, size_t n_rot)
{
    size_t half = n_rot / 2;
    for (size_t i = 0; i < half; i++) {
        float freq = powf(theta, -2.0f * (float)i / (float)n_rot);
        float ang = (float)pos * freq;
        float s = sinf(ang), c = cosf(ang);
        float a = x[2 * i], b = x[2 * i + 1];
        x[2 * i] = a * c - b * s;
        x[2 * i + 1] = a * s + b * c;
    }
}

/* crates/soso-llm-core/src/gemm.rs:62-91 (softmax_inplace + topk_softmax):
 * softmax over all, stable sort by weight desc, keep k, renormalise. */
OR_API void or_topk_softmax(float *logits, size_t n, size_t k, int32_t *idx, float *w)
{
    float mx = -INFINITY, sum = 0.0f;
    for (size_t i = 0; i < n; i++) mx = fmaxf(mx, logits[i]);
    for (size_t i = 0; i < n; i++) {
        logits[i] = expf(logits[i] - mx);
        sum += logits[i];
    }
    if (sum > 0.0f)
        for (size_t i = 0; i < n; i++) logits[i] /= sum;
    /* stable selection of the k largest (ties keep the lower index first) */
    if (k > n) k = n;
    unsigned char *used = (unsigned char *)calloc(n, 1);
    for (size_t r = 0; r < k; r++) {
        size_t best = n;
        for (size_t i = 0; i < n; i++) {
            if (used[i]) continue;
            if (best == n || logits[i] > logits[best]) best = i;
        }
        used[best] = 1;
        idx[r] = (int32_t)best;
        w[r] = logits[best];
    }
    free(used);
    float t = 0.0f;
    for (size_t r = 0; r < k; r++) t += w[r];
    if (t > 0.0f)
        for (size_t r = 0; r < k; r++) w[r] /= t;
}

/* crates/soso-llm-core/src/gemm.rs:210-226 (silu, swiglu_inplace scalar path). */
OR_API void or_swiglu(float *up, const float *gate, size_t n)
{
    for (size_t i = 0; i < n; i++) up[i] = (gate[i] / (1.0f + expf(-gate[i]))) * up[i];
}

/* crates/soso-llm-core/src/attn.rs:73-140 (attention_decode_f16_tiled_scalar):
 * online softmax over tiles of 64 positions, f16 K/V rows [token][kv_dim]. */
OR_API void or_attention_decode_f16(const float *q, const uint16_t *k, const uint16_t *v, size_t hd,
                                    size_t kv_dim, size_t kv_head, size_t n_tokens, float *out)
{
    enum { TILE = 64 };
    for (size_t d = 0; d < hd; d++) out[d] = 0.0f;
    if (n_tokens == 0 || hd == 0) return;
    float inv = 1.0f / sqrtf((float)hd), m = -INFINITY, l = 0.0f, sc[TILE];
    for (size_t t0 = 0; t0 < n_tokens; t0 += TILE) {
        size_t t1 = t0 + TILE < n_tokens ? t0 + TILE : n_tokens;
        float tmax = -INFINITY;
        for (size_t t = t0; t < t1; t++) {
            size_t off = t * kv_dim + kv_head * hd;
            float dot = 0.0f;
            for (size_t d = 0; d < hd; d++) dot += q[d] * or_f16_to_f32(k[off + d]);
            float s = dot * inv;
            sc[t - t0] = s;
            if (s > tmax) tmax = s;
        }
        float mnew = m > tmax ? m : tmax;
        float alpha = m == -INFINITY ? 0.0f : expf(m - mnew);
        for (size_t d = 0; d < hd; d++) out[d] *= alpha;
        l *= alpha;
        float ts = 0.0f;
        for (size_t t = t0; t < t1; t++) {
            float p = expf(sc[t - t0] - mnew);
            ts += p;
            size_t off = t * kv_dim + kv_head * hd;
            for (size_t d = 0; d < hd; d++) out[d] += p * or_f16_to_f32(v[off + d]);
        }
        l += ts;
        m = mnew;
    }
    if (l > 0.0f) {
        float il = 1.0f / l;
        for (size_t d = 0; d < hd; d++) out[d] *= il;
    }
}

/* crates/soso-llm-core/src/runtime.rs:2021-2028 (argmax: max_by keeps the last of equal maxima). */
OR_API int32_t or_argmax(const float *v, size_t n)
{
    size_t bi = 0;
    for (size_t i = 1; i < n; i++)
        if (!(v[i] < v[bi])) bi = i;  /* >= : later equal values win */
    return n ? (int32_t)bi : 0;
}
