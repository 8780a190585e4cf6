// engine.cuh -- whole-token decode on the device: the model resident in HBM,
// one CUDA graph per token, positions and tokens read from device memory.
//
// The boundary is GpuDispatch::decode_preparar / decode_token
// (crates/soso-llm-core/src/gpu.rs:654-684) with the plan of gpu.rs:92-158.
// One token runs the reference's dense GQA layer (layer.rs:947-1398):
//   xn = rmsnorm(h, attn_norm)                         gemm.rs:93-100
//   q|k|v = W{q,k,v} . xn  (+ bias, QK-norm, RoPE)      layer.rs:1100-1193
//   append f16 K/V at pos; o = attention(q, K, V)      kv.rs:258-275, attn.rs:73-140
//   h += Wo . o ; xn = rmsnorm(h, ffn_norm)            layer.rs:1283-1311
//   h += Wdown . (silu(Wgate . xn) * (Wup . xn))        layer.rs:1352-1389
// then logits = lm_head . rmsnorm(h, final_norm) and, for greedy decoding,
// token = argmax(logits) (runtime.rs:1976-2028).  The residual add of each
// block is fused into the RMSNorm that follows it.
//
// Per token: 5 launches per layer + 2, all captured once.  Independent matvecs
// of one input (q/k/v, gate/up) share one launch (sbk_matvec_batch_x), and the
// elementwise steps are folded into the launches around them: the residual add
// and RMSNorm into the preparation of the next matvec's input, SwiGLU into the
// down projection's, bias / QK-norm / RoPE / KV append into attention, and the
// end of a greedy step into argmax.  The residual stream alternates between two
// buffers (a matvec's CTAs read one while CTA 0 writes the other).
#pragma once
#include <algorithm>
#include <vector>

#include "dispatch.cuh"
#include "decode_ops.cuh"

extern "C" int sbk_embed_row(const void *table, uint8_t dtype, size_t vocab, size_t hidden, const int32_t *token,
                             float *out, int pdl, void *stream);
extern "C" int sbk_rope_kv_append(float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                  uint16_t *kcache, uint16_t *vcache, const int32_t *pos, size_t heads,
                                  size_t kv_heads, size_t head_dim, size_t ctx, float theta, float eps, int neox,
                                  int pdl, void *stream);
extern "C" size_t sbk_attn_ws_bytes(size_t heads, size_t kv_heads, size_t head_dim, size_t ctx);
extern "C" int sbk_attn_decode(const float *q, const uint16_t *kcache, const uint16_t *vcache, float *out,
                               const int32_t *pos, size_t heads, size_t kv_heads, size_t head_dim, size_t ctx,
                               void *ws, int pdl, void *stream);
extern "C" size_t sbk_argmax_ws_bytes(void);
extern "C" int sbk_argmax(const float *v, size_t n, int32_t *out, void *ws, int pdl, void *stream);
extern "C" int sbk_attn_rope_decode(const float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                    uint16_t *kcache, uint16_t *vcache, float *out, const int32_t *pos, size_t heads,
                                    size_t kv_heads, size_t head_dim, size_t ctx, float theta, float eps, int neox,
                                    void *ws, int pdl, void *stream);

namespace sb {

// silu(g) * u  (gemm.rs:210-226)
__global__ void swiglu_kernel(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ o, int n)
{
    griddep_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float x = g[i];
        o[i] = x / (1.0f + expf(-x)) * u[i];
    }
    griddep_launch();
}

// New K/V rows (at *pos) of every layer into one contiguous [layer][k | v] buffer.
struct KvRowsArgs {
    const uint16_t *const *kc;
    const uint16_t *const *vc;
    const int *kvd;
    const long long *off;
    int n_layers;
    const int *pos;
    uint16_t *out;
};

__global__ void kv_rows_kernel(KvRowsArgs a)
{
    griddep_wait();
    const int l = blockIdx.x, d = a.kvd[l], p = *a.pos;
    uint16_t *o = a.out + a.off[l];
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        o[i] = a.kc[l][(long long)p * d + i];
        o[d + i] = a.vc[l][(long long)p * d + i];
    }
}

}  // namespace sb

extern "C" int sbk_swiglu(const float *gate, const float *up, float *out, size_t n, int pdl, void *stream)
{
    if (!gate || !up || !out || n == 0 || n > (1u << 30)) return -1;
    const unsigned blocks = (unsigned)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3(blocks);
    c.blockDim = dim3(256);
    c.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    c.attrs = at;
    c.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&c, sb::swiglu_kernel, gate, up, out, (int)n) == cudaSuccess ? 0 : -4;
}

namespace {

struct EngMat {
    const void *w = nullptr;
    uint8_t dt = 0;
    size_t rows = 0, cols = 0;
};

struct EngLayer {
    EngMat q, k, v, o, g, u, d;
    size_t heads = 0, kvh = 0, hd = 0, qd = 0, kvd = 0, ffn = 0;
    float theta = 0.0f;
    int neox = 0;
    float *qn = nullptr, *kn = nullptr, *bias = nullptr, *na = nullptr, *nf = nullptr;
    uint16_t *kc = nullptr, *vc = nullptr;
};

}  // namespace

struct sb_engine {
    std::vector<EngLayer> L;
    size_t H = 0, V = 0, ctx = 0, ffn_max = 0, qkv_max = 0, kv_rows_total = 0;
    float eps = 0.0f;
    EngMat lm, emb;
    float *fnorm = nullptr;
    float *h = nullptr, *h2 = nullptr, *tmp = nullptr, *qkv = nullptr, *att = nullptr, *ob = nullptr, *gu = nullptr,
          *logits = nullptr;
    int *ints = nullptr;  // pos, tok, step, n_prompt
    int *prompt = nullptr, *hist = nullptr;
    void *attn_ws = nullptr, *am_ws = nullptr;
    uint16_t *kv_rows = nullptr;
    void *kv_meta = nullptr;
    std::vector<void *> allocs;
    cudaGraphExec_t g_tok = nullptr, g_greedy = nullptr;
    size_t launches_per_token = 0;

    void *dalloc(size_t bytes, cudaError_t *e)
    {
        void *p = nullptr;
        *e = cudaMalloc(&p, bytes ? bytes : 16);
        if (*e == cudaSuccess) allocs.push_back(p);
        return p;
    }
    ~sb_engine()
    {
        if (g_tok) cudaGraphExecDestroy(g_tok);
        if (g_greedy) cudaGraphExecDestroy(g_greedy);
        for (void *p : allocs) cudaFree(p);
    }
};

void sb_engine_free(sb_engine *e) { delete e; }

namespace {

// Resident weight of a plan matrix (uploaded on first sight under its key).
int eng_mat(sb_ctx *c, const sb_mat &m, size_t rows, size_t cols, EngMat *out, bool matvec)
{
    if (!m.key || !m.view.bytes) return fail("decode plan: matrix without key or bytes");
    if (m.rows != rows || m.cols != cols) return fail(std::string("decode plan: ") + m.key + " has an unexpected shape");
    if (matvec && !admit(&m.view, rows, cols)) return 0;
    Resident *r = nullptr;
    const int rc = c->resident(m.key, &m.view, rows, cols, &r, matvec);
    if (rc <= 0) return rc;
    out->w = r->ptr;
    out->dt = r->dev_dtype;
    out->rows = rows;
    out->cols = cols;
    return 1;
}

int upload_f32(sb_engine *e, const float *src, size_t n, float **dst)
{
    *dst = nullptr;
    if (!src) return 0;
    cudaError_t err;
    float *p = (float *)e->dalloc(n * 4, &err);
    if (err != cudaSuccess) return fail("cudaMalloc(plan vector)", err);
    if ((err = cudaMemcpy(p, src, n * 4, cudaMemcpyHostToDevice)) != cudaSuccess) return fail("cudaMemcpy(plan)", err);
    *dst = p;
    return 0;
}

bool fused_dtype(uint8_t dt) { return dt == SB_DTYPE_Q4_K || dt == SB_DTYPE_Q6_K_P; }

// The matvecs `ms` (one input vector a, outputs ys) with the input formed as xs says:
// one fused launch per dtype where the kernel has the fused input forms, else the
// input is materialised first (sbk_rmsnorm / sbk_swiglu into `tmp`).
int run_mv(sb_engine *e, const EngMat *const *ms, float *const *ys, int n, const float *a, const sbk_xsrc &xs,
           cudaStream_t s, size_t *launches)
{
    bool done[8] = {false};
    for (int i = 0; i < n; i++) {
        if (done[i]) continue;
        const uint8_t dt = ms[i]->dt;
        sbk_mv_op ops[8];
        int k = 0;
        for (int j = i; j < n; j++)
            if (!done[j] && ms[j]->dt == dt) ops[k++] = sbk_mv_op{ms[j]->w, ms[j]->rows, ms[j]->cols, a, ys[j]}, done[j] = true;
        int rc;
        if (fused_dtype(dt) || xs.mode == SBK_XS_PLAIN) {
            rc = xs.mode == SBK_XS_PLAIN ? sbk_matvec_batch(dt, ops, k, 1, s) : sbk_matvec_batch_x(dt, ops, k, &xs, 1, s);
        } else {
            const size_t cols = ops[0].cols;
            if (xs.mode == SBK_XS_NORM)
                rc = sbk_rmsnorm(a, xs.res, xs.res ? xs.h_out : nullptr, xs.norm_w, e->tmp, 1, cols, xs.eps, s);
            else
                rc = sbk_swiglu(a, xs.res, e->tmp, cols, 1, s);
            if (rc) return rc;
            *launches += 1;
            for (int j = 0; j < k; j++) ops[j].x = e->tmp;
            rc = sbk_matvec_batch(dt, ops, k, 1, s);
        }
        if (rc) return rc;
        *launches += 1;
    }
    return 0;
}

#define ENG_CHECK(x)                                                                                         \
    do {                                                                                                     \
        const int _rc = (x);                                                                                 \
        if (_rc) return fail(std::string("decode step: ") + #x + " rejected (" + std::to_string(_rc) + ")"); \
        n++;                                                                                                 \
    } while (0)
#define ENG_MV(...)                                                                                          \
    do {                                                                                                     \
        const int _rc = run_mv(e, __VA_ARGS__, s, &n);                                                        \
        if (_rc) return fail(std::string("decode step: matvec launch rejected (") + std::to_string(_rc) + ")"); \
    } while (0)

// One token, enqueued on s.  greedy: embedding row from the device token, and
// argmax (which also ends the step) at the end.
int enqueue_token(sb_engine *e, cudaStream_t s, bool greedy)
{
    size_t n = 0;
    int *pos = e->ints, *tok = e->ints + 1, *step = e->ints + 2, *np = e->ints + 3;
    float *hc = e->h, *ho = e->h2;  // residual stream: current / the other buffer
    if (greedy) ENG_CHECK(sbk_embed_row(e->emb.w, e->emb.dt, e->V, e->H, tok, e->h, 1, s));
    for (size_t l = 0; l < e->L.size(); l++) {
        EngLayer &L = e->L[l];
        // attention block: h (+ previous down output) -> rmsnorm -> q|k|v
        {
            const sbk_xsrc xs{l ? e->ob : nullptr, L.na, l ? ho : nullptr, e->eps, SBK_XS_NORM};
            const EngMat *ms[3] = {&L.q, &L.k, &L.v};
            float *ys[3] = {e->qkv, e->qkv + L.qd, e->qkv + L.qd + L.kvd};
            ENG_MV(ms, ys, 3, hc, xs);
            if (l) std::swap(hc, ho);
        }
        ENG_CHECK(sbk_attn_rope_decode(e->qkv, L.bias, L.qn, L.kn, L.kc, L.vc, e->att, pos, L.heads, L.kvh, L.hd,
                                       e->ctx, L.theta, e->eps, L.neox, e->attn_ws, 1, s));
        {
            const sbk_xsrc xs{nullptr, nullptr, nullptr, 0.0f, SBK_XS_PLAIN};
            const EngMat *ms[1] = {&L.o};
            float *ys[1] = {e->ob};
            ENG_MV(ms, ys, 1, e->att, xs);
        }
        // FFN block: h + attention output -> rmsnorm -> gate|up; silu(gate) * up -> down
        {
            const sbk_xsrc xs{e->ob, L.nf, ho, e->eps, SBK_XS_NORM};
            const EngMat *ms[2] = {&L.g, &L.u};
            float *ys[2] = {e->gu, e->gu + L.ffn};
            ENG_MV(ms, ys, 2, hc, xs);
            std::swap(hc, ho);
        }
        {
            const sbk_xsrc xs{e->gu + L.ffn, nullptr, nullptr, 0.0f, SBK_XS_SWIGLU};
            const EngMat *ms[1] = {&L.d};
            float *ys[1] = {e->ob};
            ENG_MV(ms, ys, 1, e->gu, xs);
        }
    }
    {
        const sbk_xsrc xs{e->ob, e->fnorm, nullptr, e->eps, SBK_XS_NORM};
        const EngMat *ms[1] = {&e->lm};
        float *ys[1] = {e->logits};
        ENG_MV(ms, ys, 1, hc, xs);
    }
    if (greedy) {
        ENG_CHECK(sb::argmax_launch(e->logits, e->V, tok, e->am_ws, 1, s, pos, step, e->hist, e->prompt, np));
    } else {
        const sb::KvRowsArgs a{(const uint16_t *const *)e->kv_meta,
                               (const uint16_t *const *)e->kv_meta + e->L.size(),
                               (const int *)((const uint16_t *const *)e->kv_meta + 2 * e->L.size()),
                               (const long long *)((const char *)e->kv_meta + 2 * e->L.size() * 8 +
                                                   ((e->L.size() * 4 + 7) & ~(size_t)7)),
                               (int)e->L.size(), pos, e->kv_rows};
        sb::kv_rows_kernel<<<(unsigned)e->L.size(), 256, 0, s>>>(a);
        if (cudaGetLastError() != cudaSuccess) return fail("decode step: kv rows launch failed");
        n++;
    }
    e->launches_per_token = n;
    return 0;
}

int capture(sb_engine *e, cudaStream_t s, bool greedy, cudaGraphExec_t *out)
{
    cudaGraph_t g = nullptr;
    cudaError_t err = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (err != cudaSuccess) return fail("cudaStreamBeginCapture", err);
    const int rc = enqueue_token(e, s, greedy);
    err = cudaStreamEndCapture(s, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (err != cudaSuccess) return fail("cudaStreamEndCapture", err);
    err = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (err != cudaSuccess) return fail("cudaGraphInstantiate", err);
    return 0;
}

}  // namespace

extern "C" int sb_decode_prepare(sb_ctx *c, const sb_decode_plan *p)
{
    if (!c || !p) return fail("null argument");
    if (!p->layers || !p->n_layers || !p->hidden || !p->vocab || !p->ctx || !p->final_norm)
        return fail("decode plan: incomplete");
    if (p->ctx > (1u << 24)) return fail("decode plan: ctx too large");
    std::lock_guard<std::mutex> lk(c->mu);
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    if (c->eng) {
        cudaStreamSynchronize(c->stream);
        sb_engine_free(c->eng);
        c->eng = nullptr;
    }
    sb_engine *e = new sb_engine();
    auto bail = [&](int rc) {
        delete e;
        return rc;
    };
    e->H = p->hidden;
    e->V = p->vocab;
    e->ctx = p->ctx;
    e->eps = p->eps;
    const size_t H = e->H;
    size_t attn_ws = 0;
    e->L.resize(p->n_layers);
    for (size_t l = 0; l < p->n_layers; l++) {
        const sb_layer_plan &lp = p->layers[l];
        EngLayer &L = e->L[l];
        if (lp.moe) return bail(0);  // MoE layers: not run by this engine
        if (!lp.norm_attn || !lp.norm_ffn) return bail(fail("decode plan: layer without norms"));
        L.heads = lp.heads, L.kvh = lp.kv_heads, L.hd = lp.head_dim, L.theta = lp.theta, L.neox = lp.neox;
        if (!L.heads || !L.kvh || L.heads % L.kvh || L.hd != 128) return bail(0);
        L.qd = L.heads * L.hd, L.kvd = L.kvh * L.hd, L.ffn = lp.gate.rows;
        int rc;
        if ((rc = eng_mat(c, lp.q, L.qd, H, &L.q, true)) != 1) return bail(rc);
        if ((rc = eng_mat(c, lp.k, L.kvd, H, &L.k, true)) != 1) return bail(rc);
        if ((rc = eng_mat(c, lp.v, L.kvd, H, &L.v, true)) != 1) return bail(rc);
        if ((rc = eng_mat(c, lp.o, H, L.qd, &L.o, true)) != 1) return bail(rc);
        if ((rc = eng_mat(c, lp.gate, L.ffn, H, &L.g, true)) != 1) return bail(rc);
        if ((rc = eng_mat(c, lp.up, L.ffn, H, &L.u, true)) != 1) return bail(rc);
        if ((rc = eng_mat(c, lp.down, H, L.ffn, &L.d, true)) != 1) return bail(rc);
        if (upload_f32(e, lp.norm_attn, H, &L.na) || upload_f32(e, lp.norm_ffn, H, &L.nf) ||
            upload_f32(e, lp.q_norm, L.hd, &L.qn) || upload_f32(e, lp.k_norm, L.hd, &L.kn) ||
            upload_f32(e, lp.qkv_bias, L.qd + 2 * L.kvd, &L.bias))
            return bail(-1);
        L.kc = (uint16_t *)e->dalloc(e->ctx * L.kvd * 2, &err);
        if (err == cudaSuccess) L.vc = (uint16_t *)e->dalloc(e->ctx * L.kvd * 2, &err);
        if (err != cudaSuccess) return bail(fail("cudaMalloc(kv cache)", err));
        e->ffn_max = std::max(e->ffn_max, L.ffn);
        e->qkv_max = std::max(e->qkv_max, L.qd + 2 * L.kvd);
        e->kv_rows_total += 2 * L.kvd;
        attn_ws = std::max(attn_ws, sbk_attn_ws_bytes(L.heads, L.kvh, L.hd, e->ctx));
    }
    int rc;
    if ((rc = eng_mat(c, p->lm_head, e->V, H, &e->lm, true)) != 1) return bail(rc);
    if (p->embed.view.bytes) {
        if (!sbk_row_bytes(p->embed.view.dtype, H) && p->embed.view.dtype != SB_DTYPE_F32) return bail(0);
        if ((rc = eng_mat(c, p->embed, e->V, H, &e->emb, false)) != 1) return bail(rc);
    }
    if (upload_f32(e, p->final_norm, H, &e->fnorm)) return bail(-1);
    // activations (each padded to 64 floats)
    auto fbuf = [&](size_t n) { return (float *)e->dalloc(((n + 63) & ~(size_t)63) * 4, &err); };
    e->h = fbuf(H);
    e->h2 = fbuf(H);
    e->qkv = fbuf(e->qkv_max);
    e->att = fbuf(e->qkv_max);
    e->ob = fbuf(H);
    e->gu = fbuf(2 * e->ffn_max);
    e->tmp = fbuf(std::max(e->ffn_max, std::max(H, e->qkv_max)));
    e->logits = fbuf(e->V);
    e->ints = (int *)e->dalloc(64, &err);
    e->prompt = (int *)e->dalloc(e->ctx * 4, &err);
    e->hist = (int *)e->dalloc(e->ctx * 4, &err);
    e->attn_ws = e->dalloc(attn_ws, &err);
    e->am_ws = e->dalloc(sbk_argmax_ws_bytes(), &err);
    e->kv_rows = (uint16_t *)e->dalloc(e->kv_rows_total * 2, &err);
    const size_t nl = e->L.size(), meta = 2 * nl * 8 + ((nl * 4 + 7) & ~(size_t)7) + nl * 8;
    e->kv_meta = e->dalloc(meta, &err);
    if (err != cudaSuccess) return bail(fail("cudaMalloc(decode buffers)", err));
    {
        std::vector<char> m(meta, 0);
        const uint16_t **kc = (const uint16_t **)m.data(), **vc = kc + nl;
        int *kvd = (int *)(m.data() + 2 * nl * 8);
        long long *off = (long long *)(m.data() + 2 * nl * 8 + ((nl * 4 + 7) & ~(size_t)7));
        long long o = 0;
        for (size_t l = 0; l < nl; l++) {
            kc[l] = e->L[l].kc, vc[l] = e->L[l].vc, kvd[l] = (int)e->L[l].kvd, off[l] = o;
            o += 2 * (long long)e->L[l].kvd;
        }
        if ((err = cudaMemcpy(e->kv_meta, m.data(), meta, cudaMemcpyHostToDevice)) != cudaSuccess)
            return bail(fail("cudaMemcpy(kv meta)", err));
    }
    // zeroed state; one eager token of each kind (sets kernel attributes, creates the
    // per-stream matvec workspace outside any capture), then capture, then re-zero
    auto zero_state = [&]() {
        cudaError_t z = cudaMemsetAsync(e->ints, 0, 64, c->stream);
        for (auto &L : e->L) {
            if (z == cudaSuccess) z = cudaMemsetAsync(L.kc, 0, e->ctx * L.kvd * 2, c->stream);
            if (z == cudaSuccess) z = cudaMemsetAsync(L.vc, 0, e->ctx * L.kvd * 2, c->stream);
        }
        if (z == cudaSuccess) z = cudaMemsetAsync(e->attn_ws, 0, attn_ws, c->stream);
        if (z == cudaSuccess) z = cudaMemsetAsync(e->am_ws, 0, sbk_argmax_ws_bytes(), c->stream);
        if (z == cudaSuccess) z = cudaMemsetAsync(e->h, 0, H * 4, c->stream);
        if (z == cudaSuccess) z = cudaStreamSynchronize(c->stream);
        return z;
    };
    if ((err = zero_state()) != cudaSuccess) return bail(fail("decode state reset", err));
    if ((rc = enqueue_token(e, c->stream, false))) return bail(rc);
    if (e->emb.w && (rc = enqueue_token(e, c->stream, true))) return bail(rc);
    if ((err = cudaStreamSynchronize(c->stream)) != cudaSuccess) return bail(fail("decode warm-up", err));
    if ((rc = capture(e, c->stream, false, &e->g_tok))) return bail(rc);
    if (e->emb.w && (rc = capture(e, c->stream, true, &e->g_greedy))) return bail(rc);
    if ((err = zero_state()) != cudaSuccess) return bail(fail("decode state reset", err));
    c->eng = e;
    return 1;
}

extern "C" int sb_decode_token(sb_ctx *c, const float *embed, size_t pos, float *logits, uint16_t *kv_rows)
{
    if (!c) return fail("null context");
    if (!embed || !logits) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    sb_engine *e = c->eng;
    if (!e || !e->g_tok) return 0;
    if (pos >= e->ctx) return fail("sb_decode_token: position beyond the prepared context");
    const uint64_t t0 = now_ns();
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    const size_t hb = (e->H * 4 + 255) & ~(size_t)255, lb = (e->V * 4 + 255) & ~(size_t)255;
    if (c->ensure_host_stage(hb + 256 + lb + e->kv_rows_total * 2)) return -1;
    char *hs = (char *)c->host_stage;
    memcpy(hs, embed, e->H * 4);
    *(int *)(hs + hb) = (int)pos;
    if ((err = cudaMemcpyAsync(e->h, hs, e->H * 4, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess ||
        (err = cudaMemcpyAsync(e->ints, hs + hb, 4, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(decode input)", err);
    if ((err = cudaGraphLaunch(e->g_tok, c->stream)) != cudaSuccess) return fail("cudaGraphLaunch", err);
    if ((err = cudaMemcpyAsync(hs + hb + 256, e->logits, e->V * 4, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(logits)", err);
    if (kv_rows && (err = cudaMemcpyAsync(hs + hb + 256 + lb, e->kv_rows, e->kv_rows_total * 2,
                                          cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(kv rows)", err);
    if ((err = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail("cudaStreamSynchronize", err);
    memcpy(logits, hs + hb + 256, e->V * 4);
    if (kv_rows) memcpy(kv_rows, hs + hb + 256 + lb, e->kv_rows_total * 2);
    c->stats.launches += e->launches_per_token;
    c->stats.bytes_up += e->H * 4 + 4;
    c->stats.bytes_down += e->V * 4 + (kv_rows ? e->kv_rows_total * 2 : 0);
    c->stats.total_ns += now_ns() - t0;
    return 1;
}

extern "C" int sb_decode_greedy(sb_ctx *c, const int32_t *prompt, size_t n_prompt, size_t pos, size_t n,
                                int32_t *tokens_out)
{
    if (!c) return fail("null context");
    if (!prompt || !n_prompt || !tokens_out) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    sb_engine *e = c->eng;
    if (!e || !e->g_greedy) return 0;
    if (n == 0) return 1;
    if (pos + n > e->ctx || n_prompt > e->ctx) return fail("sb_decode_greedy: beyond the prepared context");
    for (size_t i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || (size_t)prompt[i] >= e->V) return fail("sb_decode_greedy: token id out of range");
    const uint64_t t0 = now_ns();
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    const size_t pb = (n_prompt * 4 + 255) & ~(size_t)255;
    if (c->ensure_host_stage(pb + 256 + n * 4)) return -1;
    char *hs = (char *)c->host_stage;
    memcpy(hs, prompt, n_prompt * 4);
    int *ints = (int *)(hs + pb);
    ints[0] = (int)pos, ints[1] = prompt[0], ints[2] = 0, ints[3] = (int)n_prompt;
    if ((err = cudaMemcpyAsync(e->prompt, hs, n_prompt * 4, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess ||
        (err = cudaMemcpyAsync(e->ints, ints, 16, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(greedy input)", err);
    for (size_t i = 0; i < n; i++)
        if ((err = cudaGraphLaunch(e->g_greedy, c->stream)) != cudaSuccess) return fail("cudaGraphLaunch", err);
    if ((err = cudaMemcpyAsync(hs + pb + 256, e->hist, n * 4, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(tokens)", err);
    if ((err = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail("cudaStreamSynchronize", err);
    memcpy(tokens_out, hs + pb + 256, n * 4);
    c->stats.launches += e->launches_per_token * n;
    c->stats.total_ns += now_ns() - t0;
    return 1;
}
