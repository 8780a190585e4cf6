// experts.cuh -- the block-level GpuDispatch methods on host buffers: a tensor uploaded
// under its key (gemma_subir), the router of a block of tokens (router_topk), the routed
// and shared experts of a block grouped by expert (expertos_bloque) and the causal
// attention of a block over a host-mirrored KV cache (atencion_prefill)
// (crates/soso-llm-core/src/gpu.rs:365-530).  The device work is the block prefill's
// (pgemm.cuh, block.cuh): one grouped tensor-core GEMM for every expert's gate and up, one
// for the downs, f16 operands and f32 sums.
#pragma once
#include "block.cuh"

namespace sb {
namespace blk {

// silu(gate) * up of every slot as f16 operands of the down projection (swiglu_inplace,
// gemm.rs:210-226): rows [slot][2 ffn] = gate | up.
__global__ void swiglu16_rows_kernel(const float *__restrict__ gu, __half *__restrict__ act, int ffn, long long total)
{
    griddep_wait();
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long s = i / ffn, j = i % ffn;
        const float g = gu[s * 2 * ffn + j], u = gu[s * 2 * ffn + ffn + j];
        act[i] = __float2half_rn(g / (1.0f + expf(-g)) * u);
    }
    griddep_launch();
}

// sum[t] = sum over r in rank order of w[t k + r] * yd[slot(t k + r)] (slots < 0: not here).
__global__ void dest_combine_kernel(const float *__restrict__ yd, const int *__restrict__ dest_slot,
                                    const float *__restrict__ w, float *__restrict__ sum, int h, int k)
{
    griddep_wait();
    const int t = blockIdx.x;
    for (int i = threadIdx.x; i < h; i += blockDim.x) {
        float acc = 0.0f;
        for (int r = 0; r < k; r++) {
            const int s = dest_slot[t * k + r];
            if (s >= 0) acc += yd[(size_t)s * h + i] * w[t * k + r];
        }
        sum[(size_t)t * h + i] = acc;
    }
    griddep_launch();
}

}  // namespace blk
}  // namespace sb

namespace {

// carve 256-byte-aligned pieces out of one buffer
struct Carve {
    char *base;
    size_t off = 0;
    template <class T>
    T *take(size_t count)
    {
        T *p = reinterpret_cast<T *>(base + off);
        off += (count * sizeof(T) + 255) & ~(size_t)255;
        return p;
    }
};

}  // namespace

extern "C" int sb_upload(sb_ctx *c, const char *key, const sb_view *w, size_t rows, size_t cols)
{
    if (!c) return fail("null context");
    if (!key || !w) return fail("null argument");
    if (!w->bytes || w->elems != rows * cols || !rows || !cols) return 0;
    if (w->dtype != SB_DTYPE_F32 && (!kernel_dtype(w->dtype) || sbk_row_bytes(w->dtype, cols) * rows != w->len))
        return 0;
    if (w->dtype == SB_DTYPE_F32 && w->len != rows * cols * 4) return 0;
    std::lock_guard<std::mutex> lk(c->mu);
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return fail("cudaSetDevice", e);
    Resident *r = nullptr;
    return c->resident(key, w, rows, cols, &r, w->dtype != SB_DTYPE_F32);
}

extern "C" int sb_router_topk(sb_ctx *c, const char *key, const float *w, const float *xs, size_t n, size_t h,
                              size_t n_exp, size_t top_k, int32_t *idx, float *wts)
{
    if (!c) return fail("null context");
    if (!key || !w || !xs || !idx || !wts) return fail("null argument");
    if (!n || !h || !n_exp || !top_k || top_k > n_exp || top_k > 64 || n_exp > 4096 || n > (1u << 20)) return 0;
    std::lock_guard<std::mutex> lk(c->mu);
    const uint64_t t0 = now_ns();
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return fail("cudaSetDevice", e);
    const sb_view v{reinterpret_cast<const uint8_t *>(w), n_exp * h * 4, SB_DTYPE_F32, n_exp * h};
    Resident *r = nullptr;
    int rc = c->resident(key, &v, n_exp, h, &r, false);
    if (rc <= 0) return rc;
    const size_t xb = n * h * 4, lb = n * n_exp * 4, ib = n * top_k * 4;
    if (c->ensure_scratch(xb + lb + 2 * ib + 1024) || c->ensure_host_stage(xb + 2 * ib + 1024)) return -1;
    Carve cv{(char *)c->scratch};
    float *dx = cv.take<float>(n * h), *dl = cv.take<float>(n * n_exp), *dw = cv.take<float>(n * top_k);
    int *di = cv.take<int>(n * top_k);
    char *hs = (char *)c->host_stage;
    memcpy(hs, xs, xb);
    if ((e = cudaMemcpyAsync(dx, hs, xb, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(xs)", e);
    if (sb::launch_k(sb::blk::router_logits_f32_kernel, dim3((unsigned)((n_exp + 7) / 8), (unsigned)n), dim3(256), 0, 0,
                     c->stream, (const float *)r->ptr, (const float *)dx, dl, (int)n_exp, (int)h) ||
        sb::launch_k(sb::router_topk_kernel, dim3((unsigned)n), dim3(256), n_exp * 4, 1, c->stream, (const float *)dl,
                     (int)n_exp, (int)top_k, di, dw))
        return fail("sb_router_topk: launch failed");
    if ((e = cudaMemcpyAsync(hs, di, ib, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess ||
        (e = cudaMemcpyAsync(hs + ib, dw, ib, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess ||
        (e = cudaStreamSynchronize(c->stream)) != cudaSuccess)
        return fail("sb_router_topk", e);
    memcpy(idx, hs, ib);
    memcpy(wts, hs + ib, ib);
    c->stats.launches += 2;
    c->stats.bytes_up += xb;
    c->stats.bytes_down += 2 * ib;
    c->stats.total_ns += now_ns() - t0;
    return 1;
}

extern "C" int sb_experts(sb_ctx *c, const float *xs, size_t n, size_t h, size_t ffn, size_t top_k,
                          const float *weights, sb_expert_block *exps, size_t n_exps, float *sum, uint8_t *done)
{
    namespace pg = sb::pg;
    namespace blk = sb::blk;
    if (!c) return fail("null context");
    if (!xs || !weights || (!exps && n_exps) || !sum || !done) return fail("null argument");
    for (size_t i = 0; i < n_exps; i++) done[i] = 0;
    if (!n || !h || !ffn || !top_k || h % 64 || ffn % 64 || h < 256 || ffn < 256) return 0;
    std::lock_guard<std::mutex> lk(c->mu);
    const uint64_t t0 = now_ns();
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return fail("cudaSetDevice", e);
    // 1) the experts resolved here: resident gate / up / down of a GEMM format, with tokens
    struct PE {
        size_t i, base;
        Resident *w[3];
    };
    std::vector<PE> plan;
    size_t slots = 0;
    const size_t dims[3][2] = {{ffn, h}, {ffn, h}, {h, ffn}};
    for (size_t i = 0; i < n_exps; i++) {
        sb_expert_block &x = exps[i];
        if (!x.n_tokens || !x.tokens || !x.dests) continue;
        PE p{i, slots, {nullptr, nullptr, nullptr}};
        bool ok = true;
        for (int k = 0; k < 3 && ok; k++) {
            if (!x.keys[k]) {
                ok = false;
                break;
            }
            auto it = c->weights.find(x.keys[k]);
            if (it == c->weights.end()) {
                if (!x.views[k] || !x.views[k]->bytes || !x.views[k]->dtype) {
                    ok = false;
                    break;
                }
                if (!admit(x.views[k], dims[k][0], dims[k][1])) {
                    ok = false;
                    break;
                }
                const int rc = c->resident(x.keys[k], x.views[k], dims[k][0], dims[k][1], &p.w[k]);
                if (rc < 0) return rc;
                if (rc == 0) ok = false;
            } else {
                p.w[k] = it->second.ok ? &it->second : nullptr;
                ok = p.w[k] != nullptr;
            }
            ok = ok && (p.w[k]->dev_dtype == SB_DTYPE_Q4_K || p.w[k]->dev_dtype == SB_DTYPE_Q8_0_R) &&
                 p.w[k]->bytes == sbk_row_bytes(p.w[k]->dtype, dims[k][1]) * dims[k][0];
        }
        for (size_t j = 0; ok && j < x.n_tokens; j++)
            ok = x.tokens[j] < n && x.dests[j] < n * top_k;
        if (!ok) continue;
        plan.push_back(p);
        slots += x.n_tokens;
    }
    // 2) the host side of the launches: maps, tiles, output descriptors, slot tables
    std::vector<CUtensorMap> maps;
    std::vector<pg::Tile> t_gu, t_dn;
    std::vector<int> slot_tok(slots), dest_slot(n * top_k, -1);
    std::vector<uint8_t> dt_gu, dt_dn;
    for (const PE &p : plan) {
        const sb_expert_block &x = exps[p.i];
        CUtensorMap m[3];
        for (int k = 0; k < 3; k++)
            if (pg::make_wmap(&m[k], p.w[k]->dev_dtype, p.w[k]->ptr, (int)dims[k][0], (int)dims[k][1]))
                return fail("sb_experts: weight map failed");
        const int mi = (int)maps.size();
        maps.insert(maps.end(), m, m + 3);
        for (size_t j = 0; j < x.n_tokens; j++) {
            slot_tok[p.base + j] = (int)x.tokens[j];
            dest_slot[x.dests[j]] = (int)(p.base + j);
        }
        const int cnt = (int)x.n_tokens;
        for (int j = 0; j < cnt; j += 64) {
            const int nt = std::min(64, cnt - j);
            for (int r = 0; r < (int)ffn; r += pg::BM) {
                t_gu.push_back(pg::Tile{mi, 0, r, (int)p.base + j, nt, 0, 0, 0});
                t_gu.push_back(pg::Tile{mi + 1, 1, r, (int)p.base + j, nt, 0, 0, 0});
            }
            for (int r = 0; r < (int)h; r += pg::BM) t_dn.push_back(pg::Tile{mi + 2, 2, r, (int)p.base + j, nt, 0, 0, 0});
        }
        dt_gu.push_back(p.w[0]->dev_dtype), dt_gu.push_back(p.w[1]->dev_dtype), dt_dn.push_back(p.w[2]->dev_dtype);
    }
    for (size_t k = 1; k < dt_gu.size(); k++)
        if (dt_gu[k] != dt_gu[0]) return 0;  // one weight format per launch
    for (size_t k = 1; k < dt_dn.size(); k++)
        if (dt_dn[k] != dt_dn[0]) return 0;
    const size_t S = std::max<size_t>(slots, 1);
    // 3) device buffers (one scratch) and one upload
    const size_t need = (maps.size() * sizeof(CUtensorMap) + 1024) + (t_gu.size() + t_dn.size() + 8) * sizeof(pg::Tile) +
                        4 * sizeof(pg::Out) + n * h * 4 + n * h * 2 + S * h * 2 + S * 2 * ffn * 4 + S * ffn * 2 +
                        S * h * 4 + (S + n * top_k) * 4 + n * top_k * 4 + n * h * 4 + 16 * 256;
    if (c->ensure_scratch(need) || c->ensure_host_stage(need)) return -1;
    Carve cv{(char *)c->scratch};
    CUtensorMap *d_maps = cv.take<CUtensorMap>(std::max<size_t>(maps.size(), 1));
    pg::Tile *d_tgu = cv.take<pg::Tile>(std::max<size_t>(t_gu.size(), 1));
    pg::Tile *d_tdn = cv.take<pg::Tile>(std::max<size_t>(t_dn.size(), 1));
    pg::Out *d_outs = cv.take<pg::Out>(4);
    int *d_slot_tok = cv.take<int>(S), *d_dest = cv.take<int>(n * top_k);
    float *d_w = cv.take<float>(n * top_k), *d_x = cv.take<float>(n * h), *d_sum = cv.take<float>(n * h);
    __half *d_x16 = cv.take<__half>(n * h), *d_xg = cv.take<__half>(S * h), *d_act = cv.take<__half>(S * ffn);
    float *d_gu = cv.take<float>(S * 2 * ffn), *d_yd = cv.take<float>(S * h);
    const size_t up_bytes = (char *)d_x + n * h * 4 - (char *)c->scratch;  // everything up to xs goes up at once
    char *hs = (char *)c->host_stage;
    auto host = [&](const void *d) { return hs + ((const char *)d - (const char *)c->scratch); };
    memcpy(host(d_maps), maps.data(), maps.size() * sizeof(CUtensorMap));
    memcpy(host(d_tgu), t_gu.data(), t_gu.size() * sizeof(pg::Tile));
    memcpy(host(d_tdn), t_dn.data(), t_dn.size() * sizeof(pg::Tile));
    const pg::Out outs[3] = {{d_gu, (int)ffn, (int)(2 * ffn), 0, pg::OUT_F32},
                             {d_gu, (int)ffn, (int)(2 * ffn), (int)ffn, pg::OUT_F32},
                             {d_yd, (int)h, (int)h, 0, pg::OUT_F32}};
    memcpy(host(d_outs), outs, sizeof(outs));
    memcpy(host(d_slot_tok), slot_tok.data(), slots * 4);
    memcpy(host(d_dest), dest_slot.data(), n * top_k * 4);
    memcpy(host(d_w), weights, n * top_k * 4);
    memcpy(host(d_x), xs, n * h * 4);
    if ((e = cudaMemcpyAsync(c->scratch, hs, up_bytes, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(experts)", e);
    // 4) the launches: x -> f16, gathered per slot, gate | up, SwiGLU, down, combine
    size_t launches = 0;
    if (slots) {
        CUtensorMap xm_g, xm_d;
        if (pg::make_xmap(&xm_g, d_xg, (int)S, (int)h, 64, true) || pg::make_xmap(&xm_d, d_act, (int)S, (int)ffn, 64, true))
            return fail("sb_experts: X maps failed");
        const long long q4 = (long long)(n * h) / 4;
        int rc = sb::launch_k(blk::to16_kernel, dim3((unsigned)std::min<long long>((q4 + 255) / 256, 4096)), dim3(256),
                              0, 0, c->stream, (const float *)d_x, d_x16, q4);
        if (!rc)
            rc = sb::launch_k(blk::moe_gather16_kernel, dim3((unsigned)slots), dim3(128), 0, 1, c->stream,
                              (const __half *)d_x16, (const int *)d_slot_tok, d_xg, (int)slots, (int)h);
        pg::Launch lg{d_maps, d_outs, d_tgu, nullptr, (int)h}, ld{d_maps, d_outs, d_tdn, nullptr, (int)ffn};
        if (!rc) rc = pg::launch(dt_gu[0], 64, SBK_PREC_F16, xm_g, lg, (int)t_gu.size(), 1, c->stream);
        const long long tot = (long long)slots * ffn;
        if (!rc)
            rc = sb::launch_k(blk::swiglu16_rows_kernel, dim3((unsigned)std::min<long long>((tot + 255) / 256, 8192)),
                              dim3(256), 0, 1, c->stream, (const float *)d_gu, d_act, (int)ffn, tot);
        if (!rc) rc = pg::launch(dt_dn[0], 64, SBK_PREC_F16, xm_d, ld, (int)t_dn.size(), 1, c->stream);
        if (rc) return fail("sb_experts: launch failed (" + std::to_string(rc) + ")");
        launches += 5;
    }
    if (sb::launch_k(blk::dest_combine_kernel, dim3((unsigned)n), dim3(256), 0, 1, c->stream, (const float *)d_yd,
                     (const int *)d_dest, (const float *)d_w, d_sum, (int)h, (int)top_k))
        return fail("sb_experts: combine launch failed");
    launches++;
    if ((e = cudaMemcpyAsync(hs, d_sum, n * h * 4, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess ||
        (e = cudaStreamSynchronize(c->stream)) != cudaSuccess)
        return fail("sb_experts", e);
    memcpy(sum, hs, n * h * 4);
    for (const PE &p : plan) done[p.i] = 1;
    c->stats.launches += launches;
    c->stats.bytes_up += up_bytes;
    c->stats.bytes_down += n * h * 4;
    c->stats.total_ns += now_ns() - t0;
    return 1;
}

// The device mirror of one layer's f16 KV rows for sb_attention_prefill.
struct sb_kv_mirror {
    uint16_t *k = nullptr, *v = nullptr;
    size_t cap = 0, kv_dim = 0;
};
static std::mutex g_kvm_mu;
static std::unordered_map<const sb_ctx *, std::unordered_map<uint32_t, sb_kv_mirror>> g_kvm;

extern "C" int sb_attention_prefill(sb_ctx *c, uint32_t layer, const float *q, float *out, size_t n, size_t seq_before,
                                    size_t heads, size_t kv_heads, size_t hd, const uint16_t *k, const uint16_t *v,
                                    size_t *valid_rows)
{
    if (!c) return fail("null context");
    if (!q || !out || !k || !v || !valid_rows) return fail("null argument");
    if (!n || !heads || !kv_heads || heads % kv_heads ||
        !sb::blk::attn_prefill_takes((int)hd, (int)hd, (int)(heads / kv_heads)))
        return 0;
    std::lock_guard<std::mutex> lk(c->mu);
    const uint64_t t0 = now_ns();
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return fail("cudaSetDevice", e);
    const size_t kvd = kv_heads * hd, rows = seq_before + n;
    sb_kv_mirror *m;
    {
        std::lock_guard<std::mutex> g(g_kvm_mu);
        m = &g_kvm[c][layer];
    }
    if (m->kv_dim && m->kv_dim != kvd) {  // a new KV width for the layer: a new mirror
        cudaStreamSynchronize(c->stream);
        cudaFree(m->k);
        cudaFree(m->v);
        *m = sb_kv_mirror{};
    }
    // the caller's valid rows count up to seq_before: the block's own rows always go up
    // (kv_espejo, crates/soso-llm-api/src/cuda.rs:1389-1416)
    size_t valid = std::min(*valid_rows, m->cap ? seq_before : 0);
    if (rows > m->cap) {  // grow, keeping the rows the device holds
        const size_t cap = (rows + 4095) / 4096 * 4096;
        uint16_t *nk = nullptr, *nv = nullptr;
        if ((e = cudaMalloc(&nk, cap * kvd * 2)) != cudaSuccess || (e = cudaMalloc(&nv, cap * kvd * 2)) != cudaSuccess) {
            if (nk) cudaFree(nk);
            return fail("cudaMalloc(KV mirror)", e);
        }
        valid = std::min(valid, m->cap);
        if (m->k) {
            cudaStreamSynchronize(c->stream);
            if (valid) {
                cudaMemcpy(nk, m->k, valid * kvd * 2, cudaMemcpyDeviceToDevice);
                cudaMemcpy(nv, m->v, valid * kvd * 2, cudaMemcpyDeviceToDevice);
            }
            cudaFree(m->k);
            cudaFree(m->v);
        }
        m->k = nk, m->v = nv, m->cap = cap, m->kv_dim = kvd;
    }
    if (valid < rows) {
        if ((e = cudaMemcpyAsync(m->k + valid * kvd, k + valid * kvd, (rows - valid) * kvd * 2, cudaMemcpyHostToDevice,
                                 c->stream)) != cudaSuccess ||
            (e = cudaMemcpyAsync(m->v + valid * kvd, v + valid * kvd, (rows - valid) * kvd * 2, cudaMemcpyHostToDevice,
                                 c->stream)) != cudaSuccess)
            return fail("cudaMemcpyAsync(KV rows)", e);
        c->stats.bytes_up += (rows - valid) * kvd * 4;
    }
    const size_t qb = n * heads * hd * 4;
    if (c->ensure_scratch(2 * qb + 512) || c->ensure_host_stage(2 * qb + 512)) return -1;
    float *dq = (float *)c->scratch, *dout = (float *)((char *)c->scratch + ((qb + 255) & ~(size_t)255));
    char *hs = (char *)c->host_stage;
    memcpy(hs, q, qb);
    if ((e = cudaMemcpyAsync(dq, hs, qb, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(q)", e);
    sb::blk::AttnPrefillArgs a{dq, m->k, m->v, dout, (int)n, (int)seq_before, (int)heads, (int)kv_heads, (int)hd,
                               (int)hd, (int)(heads * hd), (int)kvd, (int)kvd, (int)(heads * hd),
                               1.0f / sqrtf((float)hd)};
    if (sb::blk::attn_prefill(a, c->stream)) return fail("sb_attention_prefill: launch failed");
    if ((e = cudaMemcpyAsync(hs, dout, qb, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess ||
        (e = cudaStreamSynchronize(c->stream)) != cudaSuccess)
        return fail("sb_attention_prefill", e);
    memcpy(out, hs, qb);
    *valid_rows = rows;
    c->stats.launches += 1;
    c->stats.bytes_up += qb;
    c->stats.bytes_down += qb;
    c->stats.total_ns += now_ns() - t0;
    return 1;
}

// the mirrors of a context go with it
void sb_kv_mirror_free(const sb_ctx *c)
{
    std::lock_guard<std::mutex> g(g_kvm_mu);
    auto it = g_kvm.find(c);
    if (it == g_kvm.end()) return;
    for (auto &kv : it->second) {
        if (kv.second.k) cudaFree(kv.second.k);
        if (kv.second.v) cudaFree(kv.second.v);
    }
    g_kvm.erase(it);
}
