// moe_layer.cuh -- GpuDispatch::moe_capa (crates/soso-llm-core/src/gpu.rs:426, MoeCapa
// :294-335; CudaGpu's moe_ejecutar, crates/soso-llm-api/src/cuda/capa/moe.rs:316): a whole
// Qwen3-MoE-style layer of a block of n tokens on the device -- RMSNorm, q|k|v, QK-norm,
// NeoX RoPE, the KV append into the layer's cache held on the device, causal attention, o,
// residual, RMSNorm, the f32 router, top-k, every routed expert's SwiGLU, the weighted sum
// and the residual -- with the hidden rows left on the device when the next layer goes on
// the GPU too (encadenar / continuar).
//
// The layer runs on the block-prefill path (prefill_engine.cuh: table-driven tcgen05 GEMMs,
// the tensor-core prefill attention, experts grouped by the device) over a one-layer engine
// built at the layer's first call from the tensors the caller made resident with sb_upload
// (gemma_subir): attention matrices by key, experts as `{prefix}.E{nn}.ffn_{gate,up,down}`.
// Each expert's gate and up are copied once, on the device, into one matrix of 16-row group
// pairs, whose GEMM forms silu(gate) * up in its epilogue.
//
// Not taken (0 = declined, the caller runs the layer on the CPU): sliding-window layers
// (ventana > 0, whose device cache evicts rows ahead), experts not resident (the streamed
// mode, ModoMoe::Flujo, fetches experts from host RAM into a pool), shapes the block path
// does not take.
#pragma once
#include <map>
#include <set>
#include <unordered_map>

#include "prefill_engine.cuh"

namespace {

struct MoeLayerState {
    sb_engine *e = nullptr;  // the layer as a one-layer engine (matrices, norms, KV cache)
    size_t stored = 0;       // KV rows the device holds (positions 0 .. stored - 1)
    size_t h = 0, heads = 0, kvh = 0, hd = 0, ffn = 0, n_exp = 0, top_k = 0, ctx = 0;
    ~MoeLayerState()
    {
        if (e) sb_engine_free(e);
    }
};

struct MoeCtxState {
    std::map<uint32_t, MoeLayerState *> layers;
    std::set<uint32_t> refused;
    float *buf[2] = {nullptr, nullptr};  // hidden rows: the input and output of a call, in turn
    size_t buf_cap = 0;                  // floats each
    int out_buf = 0;                     // buffer the last call wrote
    bool pending = false;                // a chained call's output still on the device
    uint32_t p_layer = 0;
    size_t p_pos0 = 0, p_n = 0, p_h = 0;
    ~MoeCtxState()
    {
        for (auto &kv : layers) delete kv.second;
        for (float *p : buf)
            if (p) cudaFree(p);
    }
};

std::mutex g_moe_mu;
std::unordered_map<const sb_ctx *, MoeCtxState> g_moe;

MoeCtxState &moe_state(const sb_ctx *c)
{
    std::lock_guard<std::mutex> g(g_moe_mu);
    return g_moe[c];
}

// a resident tensor (sb_upload) by key, as a GEMM operand of rows x cols
int moe_mat(sb_ctx *c, const std::string &key, size_t rows, size_t cols, EngMat *out, bool grouped = false)
{
    auto it = c->weights.find(key);
    if (it == c->weights.end() || !it->second.ok) return 0;
    const Resident &r = it->second;
    if (!sbk_row_bytes(r.dtype, cols) || r.bytes != rows * sbk_row_bytes(r.dtype, cols))
        return fail("sb_moe_layer: '" + key + "' is not a " + std::to_string(rows) + " x " + std::to_string(cols) +
                    " matrix");
    if (!(grouped ? pf_group_dtype(r.dev_dtype) : pf_gemm_dtype(r.dev_dtype))) return 0;
    *out = EngMat{r.ptr, r.dev_dtype, rows, cols};
    return 1;
}

std::string expert_key(const char *prefix, size_t e, const char *suffix)
{
    char num[24];
    snprintf(num, sizeof num, ".E%02zu.", e);
    return std::string(prefix) + num + suffix;
}

// The layer's one-layer engine: 1 = built, 0 = a shape or tensor the path does not take.
int moe_build(sb_ctx *c, const sb_moe_layer_args &a, MoeLayerState *ls)
{
    sb_engine *e = new sb_engine();
    ls->e = e;
    e->H = a.h, e->V = 0, e->ctx = a.ctx_max, e->eps = a.eps;
    e->L.resize(1);
    EngLayer &L = e->L[0];
    L.heads = a.heads, L.kvh = a.kv_heads, L.hd = a.head_dim, L.qd = a.heads * a.head_dim,
    L.kvd = a.kv_heads * a.head_dim;
    L.theta = a.theta, L.neox = 1;  // MoeCapa layers: GQA with NeoX RoPE (gpu.rs:291-293)
    L.rms = a.rope_mscale > 0.0f ? a.rope_mscale : 1.0f;
    int rc;
    if ((rc = moe_mat(c, a.key_q, L.qd, a.h, &L.q)) != 1 || (rc = moe_mat(c, a.key_k, L.kvd, a.h, &L.k)) != 1 ||
        (rc = moe_mat(c, a.key_v, L.kvd, a.h, &L.v)) != 1 || (rc = moe_mat(c, a.key_o, a.h, L.qd, &L.o)) != 1)
        return rc;
    if (L.q.dt != L.k.dt || L.q.dt != L.v.dt) return 0;  // q|k|v in one launch: one format
    if (upload_f32(e, a.attn_norm, a.h, &L.na) || upload_f32(e, a.ffn_norm, a.h, &L.nf) ||
        upload_f32(e, a.qk_norm ? a.q_norm : nullptr, a.head_dim, &L.qn) ||
        upload_f32(e, a.qk_norm ? a.k_norm : nullptr, a.head_dim, &L.kn) ||
        upload_f32(e, a.rope_factors, a.head_dim / 2, &L.rf))
        return -1;
    cudaError_t err = cudaSuccess;
    L.kc = (uint16_t *)e->dalloc(a.ctx_max * L.kvd * 2, &err);
    if (err == cudaSuccess) L.vc = (uint16_t *)e->dalloc(a.ctx_max * L.kvd * 2, &err);
    if (err != cudaSuccess) return fail("cudaMalloc(MoE layer KV cache)", err);
    // MoE FFN: the f32 router (as the reference keeps ffn_gate_inp), the experts' pair matrices
    L.moe = true, L.n_exp = a.n_exp, L.top_k = a.top_k, L.effn = a.ffn, L.ex_lo = 0, L.ex_hi = a.n_exp;
    L.ex_pairs = true;
    float *router = nullptr;
    if (upload_f32(e, a.router, a.n_exp * a.h, &router)) return -1;
    L.router = EngMat{router, SB_DTYPE_F32, a.n_exp, a.h};
    L.ex.resize(3 * a.n_exp);
    for (size_t x = 0; x < a.n_exp; x++) {
        EngMat g, u, d;
        if ((rc = moe_mat(c, expert_key(a.prefix, x, "ffn_gate"), a.ffn, a.h, &g, true)) != 1 ||
            (rc = moe_mat(c, expert_key(a.prefix, x, "ffn_up"), a.ffn, a.h, &u, true)) != 1 ||
            (rc = moe_mat(c, expert_key(a.prefix, x, "ffn_down"), a.h, a.ffn, &d, true)) != 1)
            return rc;
        if (g.dt != u.dt || (x && (g.dt != L.ex[0].dt || d.dt != L.ex[2].dt))) return 0;  // one format a kind
        if (d.dt == SB_DTYPE_Q4_K ? a.ffn % 256 != 0 : a.ffn < 256) return 0;  // the down GEMM's K
        // gate and up as 16-row group pairs, copied on the device (both resident already)
        const size_t rb = sbk_row_bytes(g.dt, a.h);
        uint8_t *p = (uint8_t *)e->dalloc(2 * a.ffn * rb + 64, &err);
        if (err != cudaSuccess) return fail("cudaMalloc(expert pairs)", err);
        const size_t grp = 16 * rb;
        if ((err = cudaMemcpy2DAsync(p, 2 * grp, g.w, grp, grp, a.ffn / 16, cudaMemcpyDeviceToDevice, c->stream)) !=
                cudaSuccess ||
            (err = cudaMemcpy2DAsync(p + grp, 2 * grp, u.w, grp, grp, a.ffn / 16, cudaMemcpyDeviceToDevice,
                                     c->stream)) != cudaSuccess)
            return fail("cudaMemcpy2DAsync(expert pairs)", err);
        L.ex[3 * x] = L.ex[3 * x + 1] = EngMat{p, g.dt, 2 * a.ffn, a.h};
        L.ex[3 * x + 2] = d;
    }
    e->ffn_max = 0, e->qkv_max = L.qd + 2 * L.kvd;
    return 1;
}

}  // namespace

extern "C" int sb_moe_layer(sb_ctx *c, sb_moe_layer_args *a)
{
    if (!c) return fail("null context");
    if (!a || !a->hidden || !a->key_q || !a->key_k || !a->key_v || !a->key_o || !a->prefix)
        return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    MoeCtxState &mc = moe_state(c);
    a->evicted = 0;
    if (mc.refused.count(a->layer)) return 0;
    if (a->cont && !(mc.pending && mc.p_layer + 1 == a->layer && mc.p_pos0 == a->pos0 && mc.p_n == a->n))
        return fail("sb_moe_layer: asked to continue from a pending output that is not the previous layer's");
    // what the block path takes (else declined, as moe_ejecutar's own checks decline)
    const size_t n = a->n, H = a->h;
    const bool shape = n > 0 && n <= 65536 && H % 256 == 0 && H <= 16384 && a->heads && a->kv_heads &&
                       a->heads % a->kv_heads == 0 && a->head_dim % 2 == 0 && (a->heads * a->head_dim) % 256 == 0 &&
                       blk::attn_prefill_takes((int)a->head_dim, (int)a->head_dim, (int)(a->heads / a->kv_heads)) &&
                       a->ffn % 64 == 0 && a->ffn >= 64 && a->n_exp >= 1 && a->n_exp <= 1024 && a->top_k >= 1 &&
                       a->top_k <= 16 && a->top_k <= a->n_exp && a->window == 0 && a->ctx_max > 0 &&
                       // the block attention scales by 1 / sqrt(head_dim), the scale the caller gives
                       // (moe_gpu.rs:236)
                       fabsf(a->scale * sqrtf((float)a->head_dim) - 1.0f) <= 1e-6f;
    if (!shape) {
        mc.refused.insert(a->layer);
        return 0;
    }
    if (a->pos0 + n > a->ctx_max)
        return fail("sb_moe_layer: " + std::to_string(a->pos0 + n) + " positions > the " +
                    std::to_string(a->ctx_max) + " held for the layer");
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    const uint64_t t0 = now_ns();
    MoeLayerState *ls = nullptr;
    {
        auto it = mc.layers.find(a->layer);
        if (it != mc.layers.end()) {
            ls = it->second;
            if (ls->h != H || ls->heads != a->heads || ls->kvh != a->kv_heads || ls->hd != a->head_dim ||
                ls->ffn != a->ffn || ls->n_exp != a->n_exp || ls->top_k != a->top_k || ls->ctx != a->ctx_max)
                return fail("sb_moe_layer: the layer's shape changed between calls");
        } else {
            if (!a->attn_norm || !a->ffn_norm || !a->router || (a->qk_norm && (!a->q_norm || !a->k_norm)))
                return fail("sb_moe_layer: the first call of a layer carries its norms and router");
            ls = new MoeLayerState();
            ls->h = H, ls->heads = a->heads, ls->kvh = a->kv_heads, ls->hd = a->head_dim, ls->ffn = a->ffn;
            ls->n_exp = a->n_exp, ls->top_k = a->top_k, ls->ctx = a->ctx_max;
            const int rc = moe_build(c, *a, ls);
            if (rc != 1) {
                cudaStreamSynchronize(c->stream);
                delete ls;
                mc.refused.insert(a->layer);
                return rc;
            }
            mc.layers[a->layer] = ls;
        }
    }
    // the layer's cache: rows up to pos0 must be there (kv_preparar_en, cuda/capa.rs:685-760)
    if (a->pos0 > ls->stored)
        return fail("sb_moe_layer: position " + std::to_string(a->pos0) + " beyond the " +
                    std::to_string(ls->stored) + " rows the device holds for layer " + std::to_string(a->layer));
    // hidden rows: in from the host, or the previous layer's output still on the device
    if (n * H > mc.buf_cap) {
        const size_t cap = std::max(n * H, 2 * mc.buf_cap);
        float *nb[2] = {nullptr, nullptr};
        if ((err = cudaMalloc(&nb[0], cap * 4)) != cudaSuccess || (err = cudaMalloc(&nb[1], cap * 4)) != cudaSuccess) {
            if (nb[0]) cudaFree(nb[0]);
            return fail("cudaMalloc(MoE layer rows)", err);
        }
        if (mc.pending && (err = cudaMemcpyAsync(nb[mc.out_buf], mc.buf[mc.out_buf], mc.p_n * H * 4,
                                                 cudaMemcpyDeviceToDevice, c->stream)) != cudaSuccess)
            return fail("cudaMemcpyAsync(pending rows)", err);
        cudaStreamSynchronize(c->stream);
        for (float *&p : mc.buf)
            if (p) cudaFree(p);
        mc.buf[0] = nb[0], mc.buf[1] = nb[1], mc.buf_cap = cap;
    }
    const int in = a->cont ? mc.out_buf : 1 - mc.out_buf, out = 1 - in;
    size_t up = 0;
    if (!a->cont) {
        // straight from the caller's (pageable) rows: the copy has read them when the call
        // returns, so the staging buffer is free for the tables the block path uploads next
        if ((err = cudaMemcpyAsync(mc.buf[in], a->hidden, n * H * 4, cudaMemcpyHostToDevice, c->stream)) !=
            cudaSuccess)
            return fail("cudaMemcpyAsync(hidden rows)", err);
        up = n * H * 4;
    }
    mc.pending = false;
    PfRun r;
    int rc = pf_run(c, ls->e, n, a->pos0, nullptr, mc.buf[in], mc.buf[out], &r);
    if (rc) return rc;
    ls->stored = a->pos0 + n;
    mc.out_buf = out;
    size_t down = 0;
    if (a->chain) {  // the next layer continues from these rows: no download, no wait
        mc.pending = true, mc.p_layer = a->layer, mc.p_pos0 = a->pos0, mc.p_n = n, mc.p_h = H;
    } else {
        if (c->ensure_host_stage(n * H * 4)) return -1;
        if ((err = cudaMemcpyAsync(c->host_stage, mc.buf[out], n * H * 4, cudaMemcpyDeviceToHost, c->stream)) !=
                cudaSuccess ||
            (err = cudaStreamSynchronize(c->stream)) != cudaSuccess)
            return fail("sb_moe_layer", err);
        memcpy(a->hidden, c->host_stage, n * H * 4);
        down = n * H * 4;
    }
    c->stats.launches += r.launches;
    c->stats.bytes_up += up + r.tiles.size() * sizeof(pg::Tile) + r.outs.size() * sizeof(pg::Out);
    c->stats.bytes_down += down;
    c->stats.total_ns += now_ns() - t0;
    return 1;
}

extern "C" int sb_moe_ready(sb_ctx *c, uint32_t layer)
{
    if (!c) return fail("null context");
    std::lock_guard<std::mutex> lk(c->mu);
    MoeCtxState &mc = moe_state(c);
    return mc.layers.count(layer) ? 1 : 0;
}

extern "C" int sb_moe_can(sb_ctx *c, uint32_t layer)
{
    if (!c) return fail("null context");
    std::lock_guard<std::mutex> lk(c->mu);
    MoeCtxState &mc = moe_state(c);
    return mc.refused.count(layer) ? 0 : 1;
}

extern "C" int sb_moe_pending(sb_ctx *c, uint32_t layer, size_t pos0, size_t n)
{
    if (!c) return fail("null context");
    std::lock_guard<std::mutex> lk(c->mu);
    MoeCtxState &mc = moe_state(c);
    return mc.pending && mc.p_layer == layer && mc.p_pos0 == pos0 && mc.p_n == n ? 1 : 0;
}

extern "C" int sb_moe_flush(sb_ctx *c, float *hidden, size_t len)
{
    if (!c) return fail("null context");
    if (!hidden) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    MoeCtxState &mc = moe_state(c);
    if (!mc.pending) return 1;
    if (len < mc.p_n * mc.p_h) return fail("sb_moe_flush: hidden shorter than the pending rows");
    const size_t bytes = mc.p_n * mc.p_h * 4;
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    if (c->ensure_host_stage(bytes)) return -1;
    if ((err = cudaMemcpyAsync(c->host_stage, mc.buf[mc.out_buf], bytes, cudaMemcpyDeviceToHost, c->stream)) !=
            cudaSuccess ||
        (err = cudaStreamSynchronize(c->stream)) != cudaSuccess)
        return fail("sb_moe_flush", err);
    memcpy(hidden, c->host_stage, bytes);
    mc.pending = false;
    c->stats.bytes_down += bytes;
    return 1;
}

extern "C" int sb_moe_discard(sb_ctx *c, uint32_t layer)
{
    if (!c) return fail("null context");
    std::lock_guard<std::mutex> lk(c->mu);
    MoeCtxState &mc = moe_state(c);
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    auto it = mc.layers.find(layer);
    if (it != mc.layers.end()) {
        delete it->second;
        mc.layers.erase(it);
    }
    mc.refused.insert(layer);
    return 1;
}

// the MoE layers of a context go with it
void sb_moe_free(const sb_ctx *c)
{
    std::lock_guard<std::mutex> g(g_moe_mu);
    g_moe.erase(c);
}
